"""The gated full-attention word step on the device (FullAttn::forward between the projections).

Mirrors crates/engine/src/model_next.rs:636-720 (FullAttn: q/k norms, rope on a quarter of each
head, the KV cache, softmax attention, the sigmoid gate) over libcwx's cwx_attn_word, for one word of
each of n_seq sequences; KvCache mirrors KvBuf (model_next.rs:61-130) without its roll: a fixed
capacity per sequence and the lengths on the device.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class FullAttn:
    """The layer's constants between the projections (model_next.rs:636-650): q_norm / k_norm
    weights (hd) and eps, n_head query heads over n_kv kv heads of dim hd, rope on the first rot
    values with base freq_base."""

    q_norm_w: torch.Tensor
    k_norm_w: torch.Tensor
    n_head: int
    n_kv: int
    hd: int
    rot: int
    freq_base: float
    eps: float

    def layer(self) -> _lib.AttnLayer:
        return _lib.AttnLayer(self.n_head, self.n_kv, self.hd, self.rot, self.eps, self.freq_base,
                              self.q_norm_w.data_ptr(), self.k_norm_w.data_ptr())


class KvCache:
    """Keys and values kept between words (KvBuf without its roll): k, v (n_seq, n_kv, cap, hd) f32
    and the rows already held per sequence, `len` (n_seq) int32 on the device."""

    def __init__(self, n_seq: int, n_kv: int, cap: int, hd: int, device):
        self.k = torch.zeros(n_seq, n_kv, cap, hd, dtype=torch.float32, device=device)
        self.v = torch.zeros_like(self.k)
        self.len = torch.zeros(n_seq, dtype=torch.int32, device=device)
        self.cap = cap


def attn_word(att: FullAttn, cache: KvCache, qg: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
              pos: torch.Tensor | None = None) -> torch.Tensor:
    """One word of every sequence: qg (n_seq, n_head, 2 hd) the wq output, k_new, v_new (n_seq, n_kv,
    hd); pos (n_seq) int32 rope positions (default: the cache lengths, the reference's offset).
    Appends the word's k, v to the cache, advances cache.len by one, and returns the gated
    attention output (n_seq, n_head * hd), the input of wo."""
    n_seq = cache.k.shape[0]
    f = lambda t: t.to(torch.float32).contiguous()  # noqa: E731
    qg, k_new, v_new = f(qg), f(k_new), f(v_new)
    if qg.numel() != n_seq * att.n_head * 2 * att.hd or k_new.numel() != n_seq * att.n_kv * att.hd:
        raise RuntimeError("coachwhip-attn-word: qg or k_new does not match the layer's heads")
    pos = cache.len.clone() if pos is None else pos.to(torch.int32).contiguous()
    out = torch.empty(n_seq, att.n_head * att.hd, dtype=torch.float32, device=qg.device)
    L = att.layer()
    dev = qg.device.index if qg.device.index is not None else torch.cuda.current_device()
    _lib.check(_lib.lib().cwx_attn_word(_lib.ctx(dev), ctypes.byref(L), n_seq, cache.cap, qg.data_ptr(),
                                        k_new.data_ptr(), v_new.data_ptr(), cache.k.data_ptr(), cache.v.data_ptr(),
                                        cache.len.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                        torch.cuda.current_stream(qg.device).cuda_stream))
    cache.len.add_(1)
    return out
