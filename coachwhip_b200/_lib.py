"""ctypes binding of libcwx.so (include/cwx.h). Loading fails loudly: there is no fallback."""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcwx.so")

OK, EINVAL, EUNSUPPORTED, ECUDA, ETIMEOUT, ENOMEM, EDEVICE, ECOMM = range(8)
TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_IQ3_S, TYPE_IQ2_S, TYPE_MXFP4 = 0, 8, 12, 14, 21, 22, 39
TYPE_IQ2_XXS, TYPE_IQ3_XXS, TYPE_IQ4_XS = 16, 18, 23
ACT_MODE_CANDLE, ACT_MODE_F32 = 0, 1
ACT_SILU, ACT_CLAMPED_SWIGLU = 0, 1
NOALLOC_SCRATCH_WORDS = 262144  # CWX_NOALLOC_SCRATCH_WORDS: cwx_permute_noalloc's fixed scratch

# Every entry point include/cwx.h declares.
EXPORTS = [
    "cwx_last_error", "cwx_version", "cwx_ctx_create", "cwx_ctx_destroy", "cwx_ctx_reserve", "cwx_ctx_status",
    "cwx_bank_create", "cwx_bank_synth", "cwx_bank_destroy", "cwx_bank_desc", "cwx_bank_download",
    "cwx_bank_dequantize", "cwx_synth_normal", "cwx_route", "cwx_permute", "cwx_permute_noalloc", "cwx_expert_matmul", "cwx_moe_forward",
    "cwx_ctx_set_profiling", "cwx_ctx_read_profile", "cwx_ctx_reset_profile", "cwx_ctx_launches",
    "cwx_ctx_set_mma_min_pile", "cwx_ep_dispatch", "cwx_ep_experts", "cwx_ep_combine", "cwx_bank_synth_experts", "cwx_bank_synth_list",
    "cwx_ep_rows_f16", "cwx_ctx_check_wait", "cwx_gguf_open", "cwx_gguf_close", "cwx_gguf_info",
    "cwx_gguf_tensor_info", "cwx_gguf_tensor", "cwx_bank_from_gguf", "cwx_gguf_tensor_f32", "cwx_gguf_meta_int",
    "cwx_gguf_meta_f64", "cwx_gguf_meta_str", "cwx_add_rms_norm", "cwx_ep_unique_id", "cwx_ep_comm_create",
    "cwx_ep_comm_wrap", "cwx_ep_comm_abort", "cwx_ep_comm_destroy", "cwx_ep_forward", "cwx_ctx_set_fused_decode",
    "cwx_gdn_word", "cwx_delta_word", "cwx_attn_word",
]
PHASES = ["router", "route", "piles", "prep", "gate_up", "down", "combine", "ep_dispatch", "ep_exchange",
          "ep_experts", "ep_return", "ep_combine", "decode_fused"]


class CwxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"cwx error {code}: {msg}")
        self.code = code


class MatrixDesc(ctypes.Structure):
    _fields_ = [("ggml_type", ctypes.c_int32), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
                ("n_experts", ctypes.c_int64), ("bytes_per_expert", ctypes.c_int64), ("host_ptr", ctypes.c_void_p)]


class MoeLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32), ("n_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("inter", ctypes.c_int32), ("norm_topk_prob", ctypes.c_int32),
        ("router_w", ctypes.c_void_p), ("router_b", ctypes.c_void_p),
        ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
        ("act", ctypes.c_int32), ("alpha", ctypes.c_float), ("limit", ctypes.c_float),
        ("gate_b", ctypes.c_void_p), ("up_b", ctypes.c_void_p), ("down_b", ctypes.c_void_p),
        ("sh_gate", ctypes.c_void_p), ("sh_up", ctypes.c_void_p), ("sh_down", ctypes.c_void_p),
        ("sh_gate_inp", ctypes.c_void_p), ("act_mode", ctypes.c_int32),
    ]


class EpGroup(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("experts_per_rank", ctypes.c_int32),
                ("placement", ctypes.c_void_p)]


class GdnLayer(ctypes.Structure):
    _fields_ = [("n_k", ctypes.c_int32), ("n_v", ctypes.c_int32), ("dk", ctypes.c_int32), ("dv", ctypes.c_int32),
                ("taps", ctypes.c_int32), ("cycle", ctypes.c_int32), ("eps", ctypes.c_float),
                ("conv_w", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p), ("a", ctypes.c_void_p),
                ("norm_w", ctypes.c_void_p)]


class AttnLayer(ctypes.Structure):
    _fields_ = [("n_head", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("hd", ctypes.c_int32), ("rot", ctypes.c_int32),
                ("eps", ctypes.c_float), ("freq_base", ctypes.c_double), ("q_norm_w", ctypes.c_void_p),
                ("k_norm_w", ctypes.c_void_p)]


class MoeArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("tokens", ctypes.c_int32), ("out", ctypes.c_void_p),
                ("residual", ctypes.c_void_p), ("ids_out", ctypes.c_void_p), ("weights_out", ctypes.c_void_p),
                ("pairs_out", ctypes.c_void_p), ("heads_out", ctypes.c_void_p),
                ("norm_w", ctypes.c_void_p), ("norm_eps", ctypes.c_float), ("norm_out", ctypes.c_void_p)]


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library; raises ImportError when libcwx.so has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python coachwhip_b200/build.py` "
                              "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        P, I32, I64, U64, F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float
        PP = ctypes.POINTER(ctypes.c_void_p)
        sig = {
            "cwx_last_error": (ctypes.c_char_p, []),
            "cwx_version": (I32, []),
            "cwx_ctx_create": (I32, [I32, PP]),
            "cwx_ctx_destroy": (I32, [P]),
            "cwx_ctx_reserve": (I32, [P, P, I32]),
            "cwx_ctx_status": (I32, [P, P]),
            "cwx_bank_create": (I32, [I32, ctypes.POINTER(MatrixDesc), PP]),
            "cwx_bank_synth": (I32, [P, I32, I64, I64, I64, U64, F, PP]),
            "cwx_bank_synth_experts": (I32, [P, I32, I64, I64, I64, I64, U64, F, PP]),
            "cwx_bank_synth_list": (I32, [P, I32, I64, I64, P, I64, U64, F, PP]),
            "cwx_bank_destroy": (I32, [P]),
            "cwx_bank_desc": (I32, [P, ctypes.POINTER(MatrixDesc)]),
            "cwx_bank_download": (I32, [P, I64, I64, P]),
            "cwx_bank_dequantize": (I32, [P, I64, P, P]),
            "cwx_synth_normal": (I32, [P, U64, U64, I64, F, P, P]),
            "cwx_route": (I32, [P, P, I32, I32, I32, I32, P, P, P]),
            "cwx_permute": (I32, [P, P, I32, I32, I32, P, P, P]),
            "cwx_permute_noalloc": (I32, [P, I32, I32, I32, P, P, P, P]),
            "cwx_expert_matmul": (I32, [P, P, P, I32, P, I32, I32, I32, P, P]),
            "cwx_moe_forward": (I32, [P, ctypes.POINTER(MoeLayer), ctypes.POINTER(MoeArgs), P]),
            "cwx_add_rms_norm": (I32, [P, P, P, P, F, I64, I32, P, P, P]),
            "cwx_ctx_set_profiling": (I32, [P, I32]),
            "cwx_ctx_read_profile": (I32, [P, P, P]),
            "cwx_ctx_reset_profile": (I32, [P]),
            "cwx_ctx_launches": (I64, [P]),
            "cwx_ctx_set_mma_min_pile": (I32, [P, I32]),
            "cwx_ep_rows_f16": (I32, [ctypes.POINTER(MoeLayer)]),
            "cwx_ctx_check_wait": (I32, [P, I32, P]),
            "cwx_ep_dispatch": (I32, [P, ctypes.POINTER(MoeLayer), ctypes.POINTER(EpGroup), P, I32, P, P, P, P, P,
                                      P, P, P]),
            "cwx_ep_experts": (I32, [P, ctypes.POINTER(MoeLayer), ctypes.POINTER(EpGroup), P, P, I32, I32, I32, P, P,
                                     P, P]),
            "cwx_ep_combine": (I32, [P, ctypes.POINTER(MoeLayer), ctypes.POINTER(EpGroup), P, I32, P, P, P, P, P, P]),
            "cwx_gguf_open": (I32, [ctypes.c_char_p, PP]),
            "cwx_gguf_close": (I32, [P]),
            "cwx_gguf_info": (I32, [P, P, P, P, P]),
            "cwx_gguf_tensor_info": (I32, [P, ctypes.c_char_p, P, P, P, P]),
            "cwx_gguf_tensor": (I32, [P, ctypes.c_char_p, ctypes.POINTER(MatrixDesc)]),
            "cwx_bank_from_gguf": (I32, [I32, P, ctypes.c_char_p, I64, I64, PP]),
            "cwx_gguf_tensor_f32": (I32, [P, ctypes.c_char_p, P, I64]),
            "cwx_gguf_meta_int": (I32, [P, ctypes.c_char_p, P]),
            "cwx_gguf_meta_f64": (I32, [P, ctypes.c_char_p, P]),
            "cwx_gguf_meta_str": (I32, [P, ctypes.c_char_p, P, I64, P]),
            "cwx_ctx_set_fused_decode": (I32, [P, I32]),
            "cwx_gdn_word": (I32, [ctypes.POINTER(GdnLayer), I32, P, P, P, P, P, P, P, P, P]),
            "cwx_delta_word": (I32, [I32, I32, I32, P, P, P, P, P]),
            "cwx_attn_word": (I32, [P, ctypes.POINTER(AttnLayer), I32, I32, P, P, P, P, P, P, P, P, P]),
            "cwx_ep_unique_id": (I32, [P, I64]),
            "cwx_ep_comm_create": (I32, [I32, P, I32, I32, PP]),
            "cwx_ep_comm_wrap": (I32, [P, I32, I32, I32, PP]),
            "cwx_ep_comm_abort": (I32, [P]),
            "cwx_ep_comm_destroy": (I32, [P]),
            "cwx_ep_forward": (I32, [P, P, ctypes.POINTER(MoeLayer), ctypes.POINTER(EpGroup), P, I32, I32, P, P, P,
                                     P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise CwxError(rc, lib().cwx_last_error().decode(errors="replace"))


_ctx: dict[tuple[int, int], ctypes.c_void_p] = {}


def ctx(device: int) -> ctypes.c_void_p:
    """This thread's context on `device` (created on first use, kept until exit)."""
    key = (device, threading.get_ident())
    c = _ctx.get(key)
    if c is None:
        c = ctypes.c_void_p()
        check(lib().cwx_ctx_create(device, ctypes.byref(c)))
        _ctx[key] = c
    return c


def status(device: int, stream: int | None = None) -> None:
    """Synchronise and raise if a kernel recorded a device-side error."""
    check(lib().cwx_ctx_status(ctx(device), stream))


def set_mma_min_pile(device: int, min_pile: int) -> None:
    """Average picks per expert from which IQ layers use the tensor-core products (0: never)."""
    check(lib().cwx_ctx_set_mma_min_pile(ctx(device), min_pile))


def set_fused_decode(device: int, max_tokens: int) -> None:
    """Batches up to max_tokens take the fused decode layer where it applies (0: never)."""
    check(lib().cwx_ctx_set_fused_decode(ctx(device), max_tokens))


def read_profile(device: int) -> tuple[list[float], list[int]]:
    """Per-phase (milliseconds, counts) recorded on this thread's context (see PHASES)."""
    ms = (ctypes.c_double * len(PHASES))()
    cnt = (ctypes.c_int64 * len(PHASES))()
    check(lib().cwx_ctx_read_profile(ctx(device), ctypes.byref(ms), ctypes.byref(cnt)))
    return list(ms), list(cnt)
