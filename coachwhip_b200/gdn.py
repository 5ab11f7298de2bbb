"""The Gated DeltaNet word step on the device: the reference's GdnWord / gdn_word and delta_word.

Mirrors crates/engine/src/attn_kernel.rs:780-895 (GdnWord, check, gdn_word) and
crates/engine/src/delta_kernel.rs:120-133 (delta_word) over libcwx's cwx_gdn_word / cwx_delta_word.
The reference runs one word of one sequence; here every per-word tensor may carry a leading batch
of n_seq independent sequences (each with its own memory and conv window), one launch for all.
Errors keep the reference's wording ("coachwhip-gdn-word: {what} must be f32, got ...").
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib


def _check(t: torch.Tensor, what: str) -> None:
    """attn_kernel.rs:797-805."""
    if t.dtype != torch.float32:
        raise RuntimeError(f"coachwhip-gdn-word: {what} must be f32, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"coachwhip-gdn-word: {what} must be contiguous")
    if not t.is_cuda:
        raise RuntimeError(f"coachwhip-gdn-word: {what} must be on a CUDA device (there is no CPU path)")


@dataclass
class GdnWord:
    """The layer's constants and this word's state (attn_kernel.rs:780-795).

    conv_state (taps-1, channels) or (n_seq, taps-1, channels); s (n_v, dk, dv) or
    (n_seq, n_v, dk, dv); conv_w (channels, taps); dt_bias, a (n_v); norm_w (dv)."""

    conv_state: torch.Tensor
    conv_w: torch.Tensor
    dt_bias: torch.Tensor
    a: torch.Tensor
    norm_w: torch.Tensor
    s: torch.Tensor
    n_k: int
    n_v: int
    dk: int
    dv: int
    taps: int
    cycle: bool
    eps: float

    def channels(self) -> int:
        return 2 * self.n_k * self.dk + self.n_v * self.dv

    def layer(self) -> _lib.GdnLayer:
        return _lib.GdnLayer(self.n_k, self.n_v, self.dk, self.dv, self.taps, 1 if self.cycle else 0, self.eps,
                             self.conv_w.data_ptr(), self.dt_bias.data_ptr(), self.a.data_ptr(),
                             self.norm_w.data_ptr())


def gdn_word(op: GdnWord, qkv: torch.Tensor, z: torch.Tensor, beta: torch.Tensor, alpha: torch.Tensor,
             s_out: torch.Tensor | None = None):
    """One word through the middle of the layer (attn_kernel.rs:880-895). Returns
    (o (n_seq, n_v*dv), s' (n_seq?, n_v, dk, dv), conv_state' (n_seq?, taps-1, channels)); with a
    single sequence and 3-dim s the shapes are the reference's ((1, n_v*dv), (n_v, dk, dv),
    (taps-1, channels)). s_out=op.s updates the memory in place."""
    for t, w in ((op.conv_state, "conv_state"), (op.conv_w, "conv_w"), (op.dt_bias, "dt_bias"), (op.a, "a"),
                 (op.norm_w, "norm_w"), (op.s, "s")):
        _check(t, w)
    n_v, dk, dv, taps = op.n_v, op.dk, op.dv, op.taps
    ch = op.channels()
    batched = op.s.dim() == 4
    n_seq = op.s.shape[0] if batched else 1
    if tuple(op.s.shape[-3:]) != (n_v, dk, dv):
        raise RuntimeError(f"coachwhip-gdn-word: s has shape {tuple(op.s.shape)}, want (.., {n_v}, {dk}, {dv})")
    if op.conv_state.numel() != n_seq * (taps - 1) * ch:
        raise RuntimeError(f"coachwhip-gdn-word: conv_state has {op.conv_state.numel()} values, "
                           f"want {n_seq} x {taps - 1} x {ch}")
    if op.conv_w.numel() != ch * taps:
        raise RuntimeError(f"coachwhip-gdn-word: conv_w has {op.conv_w.numel()} values, want {ch} x {taps}")
    f = lambda t: t.reshape(n_seq, -1).to(torch.float32).contiguous()  # noqa: E731
    qkv, z = f(qkv), f(z)
    ba = torch.cat([f(beta), f(alpha)], dim=1).contiguous()
    for t, w, n in ((qkv, "qkv", ch), (z, "z", n_v * dv), (ba, "beta/alpha", 2 * n_v)):
        _check(t, w)
        if t.shape[1] != n:
            raise RuntimeError(f"coachwhip-gdn-word: {w} has {t.shape[1]} values per word, want {n}")
    dev = qkv.device
    o = torch.empty(n_seq, n_v * dv, dtype=torch.float32, device=dev)
    if s_out is None:
        s_out = torch.empty_like(op.s)
    conv_out = torch.empty_like(op.conv_state)
    L = op.layer()
    _lib.check(_lib.lib().cwx_gdn_word(ctypes.byref(L), n_seq, qkv.data_ptr(), z.data_ptr(), ba.data_ptr(),
                                       op.conv_state.data_ptr(), op.s.data_ptr(), o.data_ptr(), s_out.data_ptr(),
                                       conv_out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
    return o, s_out, conv_out


def delta_word(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor, decay: torch.Tensor,
               s: torch.Tensor):
    """One word of the delta rule (delta_kernel.rs:120-133): q, k (n_v, dk), v (n_v, dv), beta,
    decay (n_v), s (n_v, dk, dv). Returns (o (n_v, dv), s' (n_v, dk, dv))."""
    n_v, dk, dv = s.shape
    f = lambda t: t.to(torch.float32).contiguous()  # noqa: E731
    qk = torch.cat([f(q).reshape(n_v, dk), f(k).reshape(n_v, dk)], dim=1).contiguous()
    vbd = torch.cat([f(v).reshape(n_v, dv), f(beta).reshape(n_v, 1), f(decay).reshape(n_v, 1)], dim=1).contiguous()
    s = f(s)
    for t, w in ((qk, "qk"), (vbd, "vbd"), (s, "s")):
        if not t.is_cuda:
            raise RuntimeError(f"coachwhip-delta-word: {w} must be on a CUDA device (there is no CPU path)")
    out = torch.empty(n_v, dk * dv + dv, dtype=torch.float32, device=s.device)
    _lib.check(_lib.lib().cwx_delta_word(n_v, dk, dv, qk.data_ptr(), vbd.data_ptr(), s.data_ptr(), out.data_ptr(),
                                         torch.cuda.current_stream(s.device).cuda_stream))
    return out[:, dk * dv:].contiguous(), out[:, :dk * dv].reshape(n_v, dk, dv)
