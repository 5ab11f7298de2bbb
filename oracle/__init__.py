"""CPU oracle for the MoE hot path -- TEST INFRASTRUCTURE ONLY.

ctypes wrapper around liboracle.so (C++ restatement of the reference's arithmetic, see
cw_oracle.h). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as
the checker; the product package never imports it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, Q8_0, Q4_K, Q6_K, Q8_K, IQ3_S, IQ2_S, MXFP4 = 0, 8, 12, 14, 15, 21, 22, 39
IQ2_XXS, IQ3_XXS, IQ4_XS = 16, 18, 23
MODE_CANDLE, MODE_F32 = 0, 1
ACT_SILU, ACT_CLAMPED_SWIGLU = 0, 1

_lib = None


def build() -> None:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I32, U32, U64, F = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint32,
                                    ctypes.c_uint64, ctypes.c_float)
        sig = {
            "cwo_block_elems": (I32, [I32]),
            "cwo_block_bytes": (I32, [I32]),
            "cwo_row_bytes": (I64, [I32, I64]),
            "cwo_quantize": (I32, [I32, P, I64, P]),
            "cwo_dequantize": (I32, [I32, P, I64, P]),
            "cwo_vec_dot": (F, [I32, I64, P, P]),
            "cwo_vec_dot_type": (I32, [I32]),
            "cwo_stream": (U64, [U32, U32, U32]),
            "cwo_normal": (None, [U64, U64, I64, F, P]),
            "cwo_synth_matrix": (I32, [I32, U64, I64, I64, I64, I64, F, P]),
            "cwo_router": (None, [P, P, P, I32, I32, I32, P]),
            "cwo_route": (I32, [P, I32, I32, I32, I32, P, P]),
            "cwo_router_f32": (I32, [P, P, P, I32, I32, I32, I32, P]),
            "cwo_permute": (I32, [P, I32, I32, I32, P, P]),
            "cwo_matmul": (I32, [I32, I32, P, I64, I64, I64, U32, P, I32, P]),
            "cwo_moe_forward": (I32, [P, P, I32, I32, P, P, P, P, P]),
            "cwo_add_rms_norm": (I32, [P, P, P, P, F, I64, I32, P, P]),
            "cwo_gdn_word": (I32, [I32] * 6 + [F] + [P] * 12),
            "cwo_gdn_word_ops": (I32, [I32] * 6 + [F] + [P] * 12),
            "cwo_delta_steps": (I32, [I32] * 4 + [P] * 7),
            "cwo_attn_word": (I32, [I32] * 4 + [F, ctypes.c_double] + [I32] * 3 + [P] * 8),
            "cwo_moe_forward_fast": (I32, [P, P, I32, P]),
            "cwo_set_threads": (None, [I32]),
            "cwo_get_threads": (I32, []),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def block_elems(t: int) -> int:
    return lib().cwo_block_elems(t)


def block_bytes(t: int) -> int:
    return lib().cwo_block_bytes(t)


def row_bytes(t: int, k: int) -> int:
    return lib().cwo_row_bytes(t, k)


def quantize(t: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    out = np.zeros(n // block_elems(t) * block_bytes(t), dtype=np.uint8)
    assert lib().cwo_quantize(t, _p(x), n, _p(out)) == 0
    return out


def dequantize(t: int, blocks: np.ndarray, n: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    y = np.zeros(n, dtype=np.float32)
    assert lib().cwo_dequantize(t, _p(blocks), n, _p(y)) == 0
    return y


def vec_dot(t: int, n: int, w: np.ndarray, a: np.ndarray) -> float:
    return float(lib().cwo_vec_dot(t, n, _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(a))))


def vec_dot_type(t: int) -> int:
    return lib().cwo_vec_dot_type(t)


def stream(seed: int, layer: int, tensor: int) -> int:
    return lib().cwo_stream(seed, layer, tensor)


def normal(key: int, offset: int, n: int, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().cwo_normal(key, offset, n, std, _p(out))
    return out


def synth_matrix(t: int, key: int, e0: int, ne: int, n: int, k: int, std: float) -> np.ndarray:
    out = np.empty(ne * n * row_bytes(t, k), dtype=np.uint8)
    assert lib().cwo_synth_matrix(t, key, e0, ne, n, k, std, _p(out)) == 0
    return out


def router(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    lib().cwo_router(_p(x), _p(w), _p(bb), T, H, E, _p(out))
    return out


ROUTER_ORDERS = 6  # summation orders of cwo_router_f32


def router_f32(x: np.ndarray, w: np.ndarray, b: np.ndarray | None, order: int) -> np.ndarray:
    """Router logits rounded to f32 at every step, in summation order `order` (see cw_oracle.h)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    assert lib().cwo_router_f32(_p(x), _p(w), _p(bb), T, H, E, order, _p(out)) == 0
    return out


def route(logits: np.ndarray, k: int, norm: bool) -> tuple[np.ndarray, np.ndarray]:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), dtype=np.uint32)
    w = np.empty((T, k), dtype=np.float32)
    assert lib().cwo_route(_p(logits), T, E, k, int(norm), _p(ids), _p(w)) == 0
    return ids, w


def permute(ids: np.ndarray, n_experts: int) -> tuple[np.ndarray, np.ndarray]:
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    T, k = ids.shape
    pairs = np.empty(T * k, dtype=np.uint32)
    heads = np.empty(3 * n_experts, dtype=np.uint32)
    assert lib().cwo_permute(_p(ids), T, k, n_experts, _p(pairs), _p(heads)) == 0
    return pairs, heads


def matmul(t: int, mode: int, bank: np.ndarray, n: int, k: int, bpe: int, expert: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.shape[0]
    out = np.empty((rows, n), dtype=np.float32)
    assert lib().cwo_matmul(t, mode, _p(bank), n, k, bpe, expert, _p(x), rows, _p(out)) == 0
    return out


class _Layer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int), ("n_experts", ctypes.c_int), ("top_k", ctypes.c_int),
        ("inter", ctypes.c_int), ("norm_topk_prob", ctypes.c_int),
        ("router_w", ctypes.c_void_p), ("router_b", ctypes.c_void_p),
        ("gate_type", ctypes.c_int), ("up_type", ctypes.c_int), ("down_type", ctypes.c_int),
        ("gate_bank", ctypes.c_void_p), ("up_bank", ctypes.c_void_p), ("down_bank", ctypes.c_void_p),
        ("act", ctypes.c_int), ("alpha", ctypes.c_float), ("limit", ctypes.c_float),
        ("gate_b", ctypes.c_void_p), ("up_b", ctypes.c_void_p), ("down_b", ctypes.c_void_p),
        ("shared_inter", ctypes.c_int),
        ("sh_gate_type", ctypes.c_int), ("sh_up_type", ctypes.c_int), ("sh_down_type", ctypes.c_int),
        ("sh_gate", ctypes.c_void_p), ("sh_up", ctypes.c_void_p), ("sh_down", ctypes.c_void_p),
        ("sh_gate_inp", ctypes.c_void_p),
    ]


def _layer_struct(layer: dict, keep: list) -> _Layer:

    def arr(name, dtype):
        a = layer.get(name)
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dtype)
        keep.append(a)
        return a.ctypes.data_as(ctypes.c_void_p)

    L = _Layer()
    for f in ("hidden", "n_experts", "top_k", "inter"):
        setattr(L, f, int(layer[f]))
    L.norm_topk_prob = int(layer.get("norm_topk_prob", 1))
    L.router_w = arr("router_w", np.float32)
    L.router_b = arr("router_b", np.float32)
    L.gate_type, L.up_type, L.down_type = layer["gate_type"], layer["up_type"], layer["down_type"]
    L.gate_bank, L.up_bank, L.down_bank = arr("gate_bank", np.uint8), arr("up_bank", np.uint8), arr("down_bank", np.uint8)
    L.act = int(layer.get("act", ACT_SILU))
    L.alpha = float(layer.get("alpha", 1.702))
    L.limit = float(layer.get("limit", 7.0))
    L.gate_b, L.up_b, L.down_b = arr("gate_b", np.float32), arr("up_b", np.float32), arr("down_b", np.float32)
    L.shared_inter = int(layer.get("shared_inter", 0))
    L.sh_gate_type = int(layer.get("sh_gate_type", Q4_K))
    L.sh_up_type = int(layer.get("sh_up_type", Q4_K))
    L.sh_down_type = int(layer.get("sh_down_type", Q4_K))
    L.sh_gate, L.sh_up, L.sh_down = arr("sh_gate", np.uint8), arr("sh_up", np.uint8), arr("sh_down", np.uint8)
    L.sh_gate_inp = arr("sh_gate_inp", np.float32)
    return L


def moe_forward(layer: dict, x: np.ndarray, mode: int) -> dict:
    """One MoE layer on the CPU. `layer` holds numpy arrays under the cw_oracle.h field names."""
    keep = []
    L = _layer_struct(layer, keep)
    x = np.ascontiguousarray(x, dtype=np.float32)
    T, H = x.shape
    k = L.top_k
    out = np.empty((T, H), dtype=np.float32)
    routed = np.empty((T, H), dtype=np.float32)
    shared = np.empty((T, H), dtype=np.float32)
    ids = np.empty((T, k), dtype=np.uint32)
    w = np.empty((T, k), dtype=np.float32)
    rc = lib().cwo_moe_forward(ctypes.byref(L), _p(x), T, mode, _p(out), _p(routed), _p(shared), _p(ids), _p(w))
    assert rc == 0, rc
    return {"out": out, "routed": routed, "shared": shared, "ids": ids, "w": w}


def moe_forward_fast(layer: dict, x: np.ndarray) -> np.ndarray:
    """The vectorised CPU build of the layer (candle policy, SiLU layers): the timed CPU baseline."""
    keep = []
    L = _layer_struct(layer, keep)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    rc = lib().cwo_moe_forward_fast(ctypes.byref(L), _p(x), x.shape[0], _p(out))
    assert rc == 0, rc
    return out


def add_rms_norm(a: np.ndarray, b: np.ndarray, c: np.ndarray | None, alpha: np.ndarray,
                 eps: float) -> tuple[np.ndarray, np.ndarray]:
    """(a + b (+ c), rms_norm(a + b (+ c)) * alpha) per row: add_norm with candle's CPU RmsNorm."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    c = None if c is None else np.ascontiguousarray(c, dtype=np.float32)
    alpha = np.ascontiguousarray(alpha, dtype=np.float32)
    H = a.shape[-1]
    rows = a.size // H
    s = np.empty_like(a)
    o = np.empty_like(a)
    assert lib().cwo_add_rms_norm(_p(a), _p(b), _p(c), _p(alpha), float(eps), rows, H, _p(s), _p(o)) == 0
    return s, o


def gdn_word(n_k: int, n_v: int, dk: int, dv: int, taps: int, cycle: bool, eps: float, qkv, z, ba, conv_state,
             conv_w, dt_bias, a, norm_w, s, ops: bool = False):
    """One word of one sequence through the Gated DeltaNet step: the reference's fused kernel
    (ops=False, attn_kernel.rs:24-143) or its op-by-op form (ops=True, model_next.rs:581-620).
    ba = raw beta (n_v) then raw alpha (n_v). Returns (o (n_v*dv), s' (n_v, dk, dv),
    conv_state' (taps-1, channels))."""
    f = lambda x: np.ascontiguousarray(x, dtype=np.float32)  # noqa: E731
    ch = 2 * n_k * dk + n_v * dv
    ins = [f(t) for t in (qkv, z, ba, conv_state, conv_w, dt_bias, a, norm_w, s)]
    o = np.empty(n_v * dv, np.float32)
    s_out = np.empty((n_v, dk, dv), np.float32)
    c_out = np.empty((taps - 1, ch), np.float32)
    fn = lib().cwo_gdn_word_ops if ops else lib().cwo_gdn_word
    assert fn(n_k, n_v, dk, dv, taps, int(bool(cycle)), float(eps), *[_p(t) for t in ins], _p(o), _p(s_out),
              _p(c_out)) == 0
    return o, s_out, c_out


def delta_steps(q, k, v, beta, log_decay, s):
    """The word-by-word delta rule (model_next.rs:17-38) over l words: q, k (l, n_v, dk), v (l, n_v,
    dv), beta, log_decay (l, n_v), s (n_v, dk, dv). Returns (o (l, n_v, dv), s')."""
    f = lambda x: np.ascontiguousarray(x, dtype=np.float32)  # noqa: E731
    q, k, v, beta, log_decay = f(q), f(k), f(v), f(beta), f(log_decay)
    s = np.array(s, dtype=np.float32, copy=True)
    l, n_v, dk = q.shape
    dv = v.shape[2]
    o = np.empty((l, n_v, dv), np.float32)
    assert lib().cwo_delta_steps(l, n_v, dk, dv, _p(q), _p(k), _p(v), _p(beta), _p(log_decay), _p(s), _p(o)) == 0
    return o, s


def attn_word(n_head: int, n_kv: int, hd: int, rot: int, eps: float, freq_base: float, len_: int, pos: int, qg,
              k_new, v_new, q_norm_w, k_norm_w, k_cache, v_cache):
    """One word of one sequence through the gated full attention (FullAttn::forward between the
    projections). k_cache, v_cache (n_kv, cap, hd) are copied, the new row written at len_.
    Returns (out (n_head*hd), k_cache', v_cache')."""
    f = lambda x: np.ascontiguousarray(x, dtype=np.float32)  # noqa: E731
    qg, k_new, v_new, q_norm_w, k_norm_w = f(qg), f(k_new), f(v_new), f(q_norm_w), f(k_norm_w)
    kc = np.array(k_cache, dtype=np.float32, copy=True)
    vc = np.array(v_cache, dtype=np.float32, copy=True)
    cap = kc.shape[1]
    out = np.empty(n_head * hd, np.float32)
    assert lib().cwo_attn_word(n_head, n_kv, hd, rot, float(eps), float(freq_base), cap, len_, pos, _p(qg), _p(k_new),
                               _p(v_new), _p(q_norm_w), _p(k_norm_w), _p(kc), _p(vc), _p(out)) == 0
    return out, kc, vc


def set_threads(n: int) -> None:
    lib().cwo_set_threads(n)


def get_threads() -> int:
    return lib().cwo_get_threads()
