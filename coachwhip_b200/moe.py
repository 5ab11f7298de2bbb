"""coachwhip's MoE layer API on the cwx CUDA library.

Mirrors the Rust interface of the reference's resident MoE path so a caller reads the same:
  route(logits, top_k, norm) -> (ids, weights)       crates/engine/src/experts.rs:2364-2372
  ExpertAct.Silu / ExpertAct.ClampedSwiglu(...)       experts.rs:2376-2422
  MoeMatvec(...)(x, ids)                              experts.rs:2183-2309 (CustomOp2 metal_fwd)
  ExpertStore.resident_op(layer, which, nei0, rpe)    experts.rs:1949-1998
  SharedExpert(gate_inp, gate, up, down).forward(x)   crates/engine/src/model_next.rs:723-742
  StreamedMoe(...).forward(xs)                        experts.rs:2426-2440, 2539-2614
Tensors are torch CUDA tensors (PyTorch is only the device-memory and stream plumbing); every
computation runs in libcwx.so. Errors raise CwxError (or ValueError for the checks the reference
does with candle::bail!) with the reference's wording.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import CwxError, check

BLOCK = {  # ggml type -> (elements, bytes) per quant block
    _lib.TYPE_Q8_0: (32, 34), _lib.TYPE_Q4_K: (256, 144), _lib.TYPE_Q6_K: (256, 210),
    _lib.TYPE_IQ3_S: (256, 110), _lib.TYPE_IQ2_S: (256, 82), _lib.TYPE_MXFP4: (32, 17),
    _lib.TYPE_IQ2_XXS: (256, 66), _lib.TYPE_IQ3_XXS: (256, 98), _lib.TYPE_IQ4_XS: (256, 136),
}


def row_bytes(ggml_type: int, k: int) -> int:
    be, bb = BLOCK[ggml_type]
    if k % be:
        raise ValueError(f"k={k} is not a multiple of the {be}-element block")
    return k // be * bb


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _dev_index(t: torch.Tensor) -> int:
    if t.device.type != "cuda":
        raise ValueError("coachwhip-b200 tensors must live on a CUDA device")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


class Bank:
    """One GGUF expert tensor (n_experts, n, k) resident in HBM (a cwx_bank)."""

    def __init__(self, handle: ctypes.c_void_p, ggml_type: int, n: int, k: int, n_experts: int, device: int):
        self.handle = handle
        self.ggml_type, self.n, self.k, self.n_experts, self.device = ggml_type, n, k, n_experts, device

    @classmethod
    def from_gguf_bytes(cls, data: np.ndarray, ggml_type: int, n: int, k: int, n_experts: int, device: int = 0) -> "Bank":
        data = np.ascontiguousarray(data, dtype=np.uint8)
        bpe = n * row_bytes(ggml_type, k)
        if data.size != bpe * n_experts:
            raise ValueError(f"{data.size} bytes for {n_experts} experts of {bpe}")
        d = _lib.MatrixDesc(ggml_type, n, k, n_experts, bpe, data.ctypes.data)
        h = ctypes.c_void_p()
        check(_lib.lib().cwx_bank_create(device, ctypes.byref(d), ctypes.byref(h)))
        return cls(h, ggml_type, n, k, n_experts, device)

    @classmethod
    def synth(cls, ggml_type: int, n: int, k: int, n_experts: int, key: int, std: float, device: int = 0,
              first: int = 0) -> "Bank":
        """Synthetic N(0, std^2) bank of stream `key`: experts first .. first + n_experts - 1 of it."""
        h = ctypes.c_void_p()
        check(_lib.lib().cwx_bank_synth_experts(_lib.ctx(device), ggml_type, n, k, first, n_experts, key, std,
                                                ctypes.byref(h)))
        return cls(h, ggml_type, n, k, n_experts, device)

    @classmethod
    def synth_list(cls, ggml_type: int, n: int, k: int, experts, key: int, std: float, device: int = 0) -> "Bank":
        """Synthetic bank holding the listed experts of stream `key`, in list order."""
        ids = np.ascontiguousarray(np.asarray(experts, dtype=np.int64))
        h = ctypes.c_void_p()
        check(_lib.lib().cwx_bank_synth_list(_lib.ctx(device), ggml_type, n, k, ids.ctypes.data, int(ids.size), key,
                                             std, ctypes.byref(h)))
        return cls(h, ggml_type, n, k, int(ids.size), device)

    @property
    def bytes_per_expert(self) -> int:
        return self.n * row_bytes(self.ggml_type, self.k)

    def download(self, e0: int = 0, ne: int | None = None) -> np.ndarray:
        ne = self.n_experts - e0 if ne is None else ne
        out = np.empty(ne * self.bytes_per_expert, dtype=np.uint8)
        check(_lib.lib().cwx_bank_download(self.handle, e0, ne, out.ctypes.data))
        return out

    def dequantize(self, expert: int) -> torch.Tensor:
        out = torch.empty((self.n, self.k), dtype=torch.float32, device=f"cuda:{self.device}")
        check(_lib.lib().cwx_bank_dequantize(self.handle, expert, out.data_ptr(), _stream(out.device)))
        return out

    def close(self) -> None:
        if self.handle:
            _lib.lib().cwx_bank_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def route(logits: torch.Tensor, top_k: int, norm: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """The router's choice for each token: the top_k likeliest experts, best first (ties: lowest
    id), and their softmax weights, rescaled to sum to 1 when norm. Returns (ids u32-as-int32,
    weights f32)."""
    if logits.dtype != torch.float32 or not logits.is_contiguous() or logits.dim() != 2:
        raise ValueError("route: logits must be a contiguous (tokens, experts) f32 tensor")
    t, e = logits.shape
    ids = torch.empty((t, top_k), dtype=torch.int32, device=logits.device)
    w = torch.empty((t, top_k), dtype=torch.float32, device=logits.device)
    dev = _dev_index(logits)
    check(_lib.lib().cwx_route(_lib.ctx(dev), logits.data_ptr(), t, e, top_k, int(bool(norm)), ids.data_ptr(),
                               w.data_ptr(), _stream(logits.device)))
    return ids, w


def piles(ids: torch.Tensor, n_experts: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(pairs, heads): pick indices grouped by expert (stable) and (expert, first, count) rows."""
    t, k = ids.shape
    pairs = torch.empty(t * k, dtype=torch.int32, device=ids.device)
    heads = torch.empty((n_experts, 3), dtype=torch.int32, device=ids.device)
    dev = _dev_index(ids)
    check(_lib.lib().cwx_permute(_lib.ctx(dev), ids.data_ptr(), t, k, n_experts, pairs.data_ptr(), heads.data_ptr(),
                                 _stream(ids.device)))
    return pairs, heads


class ExpertAct:
    """What a family does between an expert's matrices."""

    @dataclass
    class Silu:
        pass

    @dataclass
    class ClampedSwiglu:
        alpha: float
        limit: float
        gate_b: torch.Tensor | None
        up_b: torch.Tensor | None
        down_b: torch.Tensor | None
        pad: int = 0


@dataclass
class MoeMatvec:
    """x (rows, k), ids (tokens, nei0) -> (tokens, nei0, n): each token's picks times their
    expert's matrix; with rows_per_expert x has one row per (token, pick)."""

    bank: Bank
    nei0: int
    rows_per_expert: bool
    act_mode: int = _lib.ACT_MODE_CANDLE

    def __call__(self, x: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        if not x.is_contiguous() or not ids.is_contiguous():
            raise ValueError("coachwhip-moe-matvec needs contiguous inputs")
        if x.dtype != torch.float32 or ids.dtype not in (torch.int32, torch.uint32):
            raise ValueError("coachwhip-moe-matvec: x must be f32 and ids u32")
        tokens, nei0 = ids.shape
        if nei0 != self.nei0:
            raise ValueError(f"coachwhip-moe-matvec: {nei0} ids per token, expected {self.nei0}")
        rows, k = x.shape
        if k != self.bank.k or rows != (tokens * nei0 if self.rows_per_expert else tokens):
            raise ValueError(f"coachwhip-moe-matvec: x is {rows}x{k}, expected k={self.bank.k} for {tokens} tokens")
        out = torch.empty((tokens, nei0, self.bank.n), dtype=torch.float32, device=x.device)
        dev = _dev_index(x)
        check(_lib.lib().cwx_expert_matmul(_lib.ctx(dev), self.bank.handle, x.data_ptr(), int(self.rows_per_expert),
                                           ids.data_ptr(), tokens, nei0, self.act_mode, out.data_ptr(),
                                           _stream(x.device)))
        return out


class ExpertStore:
    """Every layer's expert banks resident in HBM: (gate, up, down) per layer."""

    def __init__(self, banks: list[tuple[Bank, Bank, Bank]]):
        self.banks = banks

    def resident_op(self, layer: int, which: int, nei0: int, rows_per_expert: bool,
                    act_mode: int = _lib.ACT_MODE_CANDLE) -> MoeMatvec:
        return MoeMatvec(self.banks[layer][which], nei0, rows_per_expert, act_mode)


@dataclass
class SharedExpert:
    """The expert every token uses, gated by sigmoid(x . gate_inp)."""

    gate_inp: torch.Tensor  # (hidden,) f32
    gate: Bank
    up: Bank
    down: Bank


class StreamedMoe:
    """One MoE layer whose experts live in the ExpertStore (all resident)."""

    def __init__(self, layer: int, gate: torch.Tensor, top_k: int, norm_topk_prob: bool, act, store: ExpertStore,
                 gate_bias: torch.Tensor | None = None, shared: SharedExpert | None = None,
                 act_mode: int = _lib.ACT_MODE_CANDLE):
        self.layer, self.gate, self.gate_bias = layer, gate.contiguous(), gate_bias
        self.top_k, self.norm_topk_prob, self.act, self.store = top_k, norm_topk_prob, act, store
        self.shared, self.act_mode = shared, act_mode
        g, u, d = store.banks[layer]
        self.n_experts, self.hidden = gate.shape
        self.inter = g.n
        L = _lib.MoeLayer()
        L.hidden, L.n_experts, L.top_k, L.inter = self.hidden, self.n_experts, top_k, self.inter
        L.norm_topk_prob = int(bool(norm_topk_prob))
        L.router_w = self.gate.data_ptr()
        L.router_b = _ptr(gate_bias)
        L.gate, L.up, L.down = g.handle, u.handle, d.handle
        if isinstance(act, ExpertAct.ClampedSwiglu):
            L.act, L.alpha, L.limit = _lib.ACT_CLAMPED_SWIGLU, float(act.alpha), float(act.limit)
            L.gate_b, L.up_b, L.down_b = _ptr(act.gate_b), _ptr(act.up_b), _ptr(act.down_b)
        else:
            L.act = _lib.ACT_SILU
        if shared is not None:
            L.sh_gate, L.sh_up, L.sh_down = shared.gate.handle, shared.up.handle, shared.down.handle
            L.sh_gate_inp = shared.gate_inp.data_ptr()
        L.act_mode = act_mode
        self._layer = L

    def forward(self, xs: torch.Tensor, residual: torch.Tensor | None = None, taps: dict | None = None) -> torch.Tensor:
        """xs (b, s, h) -> routed experts (+ shared expert when configured, + residual when given),
        in the input's dtype; the layer computes in f32 as the reference does."""
        b, s, h = xs.shape
        n = b * s
        dtype = xs.dtype
        x = xs.reshape(n, h).to(torch.float32).contiguous()
        out = torch.empty((n, h), dtype=torch.float32, device=xs.device)
        A = _lib.MoeArgs()
        A.x, A.tokens, A.out = x.data_ptr(), n, out.data_ptr()
        res = None
        if residual is not None:
            res = residual.reshape(n, h).to(torch.float32).contiguous()
            A.residual = res.data_ptr()
        if taps is not None:
            taps["ids"] = torch.empty((n, self.top_k), dtype=torch.int32, device=xs.device)
            taps["weights"] = torch.empty((n, self.top_k), dtype=torch.float32, device=xs.device)
            taps["pairs"] = torch.empty(n * self.top_k, dtype=torch.int32, device=xs.device)
            taps["heads"] = torch.empty((self.n_experts, 3), dtype=torch.int32, device=xs.device)
            A.ids_out, A.weights_out = taps["ids"].data_ptr(), taps["weights"].data_ptr()
            A.pairs_out, A.heads_out = taps["pairs"].data_ptr(), taps["heads"].data_ptr()
        dev = _dev_index(xs)
        check(_lib.lib().cwx_moe_forward(_lib.ctx(dev), ctypes.byref(self._layer), ctypes.byref(A), _stream(xs.device)))
        return out.reshape(b, s, h).to(dtype)

    def forward_norm(self, xs: torch.Tensor, residual: torch.Tensor | None, norm_w: torch.Tensor,
                     eps: float) -> tuple[torch.Tensor, torch.Tensor]:
        """forward() with the reference's residual step fused after the combine (add_norm,
        crates/engine/src/model_next.rs:1432-1436): returns (out, rms_norm(out) * norm_w), out as
        forward() gives it (f32), the second the next layer's normalised input."""
        b, s, h = xs.shape
        n = b * s
        if norm_w.dtype != torch.float32 or norm_w.shape != (h,):
            raise ValueError(f"add_norm: f32 ({h},) norm weight expected, got {norm_w.dtype} {tuple(norm_w.shape)}")
        x = xs.reshape(n, h).to(torch.float32).contiguous()
        out = torch.empty((n, h), dtype=torch.float32, device=xs.device)
        normed = torch.empty((n, h), dtype=torch.float32, device=xs.device)
        w = norm_w.contiguous()
        A = _lib.MoeArgs()
        A.x, A.tokens, A.out = x.data_ptr(), n, out.data_ptr()
        res = None
        if residual is not None:
            res = residual.reshape(n, h).to(torch.float32).contiguous()
            A.residual = res.data_ptr()
        A.norm_w, A.norm_eps, A.norm_out = w.data_ptr(), float(eps), normed.data_ptr()
        check(_lib.lib().cwx_moe_forward(_lib.ctx(_dev_index(xs)), ctypes.byref(self._layer), ctypes.byref(A),
                                         _stream(xs.device)))
        return out.reshape(b, s, h), normed.reshape(b, s, h)

    def reserve(self, tokens: int) -> None:
        """Size the workspace for `tokens` (before capturing forward() in a CUDA graph)."""
        check(_lib.lib().cwx_ctx_reserve(_lib.ctx(self.gate.device.index or 0), ctypes.byref(self._layer), tokens))


def add_norm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor | None, alpha: torch.Tensor,
             eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(a + b (+ c), rms_norm(a + b (+ c)) * alpha) in one launch: fuse_kernel::add_norm
    (crates/engine/src/fuse_kernel.rs:433-471), with the same checks (f32 only, alpha the last
    dimension's size)."""
    ts = [a, b, alpha] + ([c] if c is not None else [])
    if any(t.dtype != torch.float32 for t in ts):
        raise ValueError("add_norm: f32 only")
    h = a.shape[-1]
    if b.shape != a.shape or (c is not None and c.shape != a.shape) or alpha.shape != (h,):
        raise ValueError(f"add_norm: shapes {tuple(a.shape)}, {tuple(b.shape)}, alpha {tuple(alpha.shape)}")
    if any(t.device != a.device for t in ts) or a.device.type != "cuda":
        raise ValueError("add_norm: all tensors on one CUDA device")
    a, b, alpha = a.contiguous(), b.contiguous(), alpha.contiguous()
    c = c.contiguous() if c is not None else None
    s = torch.empty_like(a)
    o = torch.empty_like(a)
    check(_lib.lib().cwx_add_rms_norm(a.data_ptr(), b.data_ptr(), _ptr(c), alpha.data_ptr(), float(eps),
                                      a.numel() // h, h, s.data_ptr(), o.data_ptr(), _stream(a.device)))
    return s, o


__all__ = ["Bank", "route", "piles", "add_norm", "ExpertAct", "MoeMatvec", "ExpertStore", "SharedExpert", "StreamedMoe",
           "CwxError", "row_bytes"]
