"""Expert-parallel MoE layer: experts split over the ranks of a process group.

The reference runs one device; this is the multi-GPU form of its layer (StreamedMoe::forward,
crates/engine/src/experts.rs:2539-2614) with the same output. Rank r owns experts
[r*epr, (r+1)*epr) (epr = n_experts / world) and routes its own tokens. One layer:

  1. dispatch (cwx_ep_dispatch): router, route and piles over all experts; the picks' rows in
     pile order, which groups them by the rank that owns their expert, with each pick's expert
     rewritten to its index on that rank;
  2. exchange the per-rank counts, then the rows and expert indices (all-to-all with uneven
     splits);
  3. experts (cwx_ep_experts): the received rows through this rank's experts, one pick per row;
  4. exchange the result rows back (the reverse splits), so every rank gets its picks' rows in
     the order it sent them;
  5. combine (cwx_ep_combine): weighted sum in pick order + shared expert on the local tokens +
     residual.

The exchanges use torch.distributed (NCCL between GPUs; the steps themselves run in libcwx.so).
The count exchange is read on the host to size the row exchange, so a layer synchronises once.
`Engine` is the per-rank compute; `CudaEngine` is the product, and tests substitute a CPU engine
built on the oracle to check the exchange protocol on gloo ranks.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check
from .moe import Bank, ExpertAct, SharedExpert, _dev_index, _ptr, _stream


@dataclass
class Dispatched:
    """What step 1 leaves for step 5 and the rows it sends."""

    x: torch.Tensor          # (T, H) f32 local tokens
    weights: torch.Tensor    # (T, k) f32
    pairs: torch.Tensor      # (T*k,) pile order of the picks
    sgate: torch.Tensor | None
    send_rows: torch.Tensor  # (T*k, H) f32
    send_eids: torch.Tensor  # (T*k,) int32 expert index on the destination rank
    send_counts: torch.Tensor  # (world,) int32


class CudaEngine:
    """This rank's steps on its GPU through libcwx.so."""

    def __init__(self, gate: torch.Tensor, top_k: int, norm_topk_prob: bool, act, banks: tuple[Bank, Bank, Bank],
                 world: int, rank: int, gate_bias: torch.Tensor | None = None, shared: SharedExpert | None = None,
                 act_mode: int = _lib.ACT_MODE_CANDLE):
        self.gate, self.gate_bias, self.shared = gate.contiguous(), gate_bias, shared
        self.n_experts, self.hidden = self.gate.shape
        if self.n_experts % world:
            raise ValueError(f"{self.n_experts} experts do not split over {world} ranks")
        self.epr = self.n_experts // world
        g, u, d = banks
        if g.n_experts != self.epr or u.n_experts != self.epr or d.n_experts != self.epr:
            raise ValueError(f"the banks must hold this rank's {self.epr} experts")
        self.top_k, self.banks, self.act = top_k, banks, act
        L = _lib.MoeLayer()
        L.hidden, L.n_experts, L.top_k, L.inter = self.hidden, self.n_experts, top_k, g.n
        L.norm_topk_prob = int(bool(norm_topk_prob))
        L.router_w = self.gate.data_ptr()
        L.router_b = _ptr(gate_bias)
        L.gate, L.up, L.down = g.handle, u.handle, d.handle
        if isinstance(act, ExpertAct.ClampedSwiglu):  # biases: this rank's experts' rows
            L.act, L.alpha, L.limit = _lib.ACT_CLAMPED_SWIGLU, float(act.alpha), float(act.limit)
            L.gate_b, L.up_b, L.down_b = _ptr(act.gate_b), _ptr(act.up_b), _ptr(act.down_b)
        else:
            L.act = _lib.ACT_SILU
        if shared is not None:
            L.sh_gate, L.sh_up, L.sh_down = shared.gate.handle, shared.up.handle, shared.down.handle
            L.sh_gate_inp = shared.gate_inp.data_ptr()
        L.act_mode = act_mode
        self._layer = L
        self._group = _lib.EpGroup(world, rank, self.epr)

    def dispatch(self, x: torch.Tensor) -> Dispatched:
        T, H = x.shape
        n = T * self.top_k
        dev = x.device
        ids = torch.empty(n, dtype=torch.int32, device=dev)
        w = torch.empty((T, self.top_k), dtype=torch.float32, device=dev)
        pairs = torch.empty(n, dtype=torch.int32, device=dev)
        sgate = torch.empty(T, dtype=torch.float32, device=dev) if self.shared is not None else None
        rows = torch.empty((n, H), dtype=torch.float32, device=dev)
        eids = torch.empty(n, dtype=torch.int32, device=dev)
        counts = torch.empty(self._group.world, dtype=torch.int32, device=dev)
        check(_lib.lib().cwx_ep_dispatch(_lib.ctx(_dev_index(x)), ctypes.byref(self._layer), ctypes.byref(self._group),
                                         x.data_ptr(), T, ids.data_ptr(), w.data_ptr(), pairs.data_ptr(), _ptr(sgate),
                                         rows.data_ptr(), eids.data_ptr(), counts.data_ptr(), _stream(dev)))
        return Dispatched(x, w, pairs, sgate, rows, eids, counts)

    def experts(self, rows: torch.Tensor, eids: torch.Tensor) -> torch.Tensor:
        n = rows.shape[0]
        y = torch.empty((n, self.hidden), dtype=torch.float32, device=rows.device)
        if n:
            check(_lib.lib().cwx_ep_experts(_lib.ctx(_dev_index(rows)), ctypes.byref(self._layer),
                                            ctypes.byref(self._group), rows.data_ptr(), eids.data_ptr(), n,
                                            y.data_ptr(), _stream(rows.device)))
        return y

    def combine(self, d: Dispatched, back: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        T, H = d.x.shape
        out = torch.empty((T, H), dtype=torch.float32, device=d.x.device)
        check(_lib.lib().cwx_ep_combine(_lib.ctx(_dev_index(d.x)), ctypes.byref(self._layer), d.x.data_ptr(), T,
                                        d.weights.data_ptr(), d.pairs.data_ptr(), back.data_ptr(), _ptr(d.sgate),
                                        _ptr(residual), out.data_ptr(), _stream(d.x.device)))
        return out


class ExpertParallelMoe:
    """One MoE layer whose experts are split over the ranks of `group` (torch.distributed)."""

    def __init__(self, engine, group=None):
        import torch.distributed as dist

        self.engine, self.group = engine, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        import torch.distributed as dist

        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, xs: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """xs (b, s, h) local tokens -> this rank's layer output, in the input's dtype."""
        b, s, h = xs.shape
        x = xs.reshape(b * s, h).to(torch.float32).contiguous()
        res = None if residual is None else residual.reshape(b * s, h).to(torch.float32).contiguous()
        d = self.engine.dispatch(x)
        # counts first: every rank learns how many rows each peer sends it
        recv_counts = torch.empty_like(d.send_counts)
        if self.world == 1:
            recv_counts.copy_(d.send_counts)
        else:
            import torch.distributed as dist

            dist.all_to_all_single(recv_counts, d.send_counts, group=self.group)
        sc = [int(v) for v in d.send_counts.tolist()]
        rc = [int(v) for v in recv_counts.tolist()]
        nr = sum(rc)
        rows = torch.empty((nr, h), dtype=torch.float32, device=x.device)
        eids = torch.empty(nr, dtype=torch.int32, device=x.device)
        self._a2a(rows, d.send_rows, rc, sc)
        self._a2a(eids, d.send_eids, rc, sc)
        y = self.engine.experts(rows, eids)
        back = torch.empty((sum(sc), h), dtype=torch.float32, device=x.device)
        self._a2a(back, y, sc, rc)
        out = self.engine.combine(d, back, res)
        return out.reshape(b, s, h).to(xs.dtype)


__all__ = ["CudaEngine", "Dispatched", "ExpertParallelMoe"]
