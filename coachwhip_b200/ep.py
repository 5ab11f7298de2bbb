"""Expert-parallel MoE layer: experts split over the ranks of a process group.

The reference runs one device; this is the multi-GPU form of its layer (StreamedMoe::forward,
crates/engine/src/experts.rs:2539-2614) with the same output. Rank r owns experts
[r*epr, (r+1)*epr) (epr = n_experts / world) and routes its own tokens. One layer:

  1. dispatch (cwx_ep_dispatch): router and route over all experts; a token's row goes once to
     each rank that owns any of its picks (a unit), with one record per pick (unit, expert index
     on that rank, weight);
  2. exchange the per-rank counts (units, records), then the rows and the records (all-to-all
     with uneven splits);
  3. experts (cwx_ep_experts): the received records through this rank's experts, each unit's
     weighted sum in record order;
  4. exchange the unit rows back (the reverse splits), so every rank gets its units in the order
     it sent them;
  5. combine (cwx_ep_combine): the units' rows summed in rank order + shared expert on the local
     tokens + residual.

ExpertParallelMoe makes the exchanges with torch.distributed (NCCL between GPUs, gloo in the CPU
protocol tests; the steps themselves run in libcwx.so); its count exchange is read on the host to
size the row exchange, so a layer synchronises once. LibraryExpertParallelMoe runs the whole layer
in cwx_ep_forward, with the library's own NCCL communicator (EpComm) and fixed-capacity exchanges
whose counts stay on the device: no host synchronisation, and no PyTorch needed by a native host.
`Engine` is the per-rank compute; `CudaEngine` is the product, and tests substitute a CPU engine
built on the oracle to check the exchange protocol on gloo ranks.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check
from .moe import Bank, ExpertAct, SharedExpert, _dev_index, _ptr, _stream


@dataclass
class Dispatched:
    """What step 1 leaves for step 5 and what it sends."""

    x: torch.Tensor           # (T, H) f32 local tokens
    ids: torch.Tensor | None  # (T, top_k) int32 expert ids of the local tokens (None: not kept)
    unit_of: torch.Tensor     # (T, world) int32: the token's unit in send_rows per rank, or -1
    sgate: torch.Tensor | None
    send_rows: torch.Tensor   # (units, H) f16 or f32, destinations in rank order
    send_picks: torch.Tensor  # (records, 3) int32: unit in its message, expert on the rank, weight bits
    send_counts: torch.Tensor  # (world, 2) int32: units, records per destination


class CudaEngine:
    """This rank's steps on its GPU through libcwx.so."""

    def __init__(self, gate: torch.Tensor, top_k: int, norm_topk_prob: bool, act, banks: tuple[Bank, Bank, Bank],
                 world: int, rank: int, gate_bias: torch.Tensor | None = None, shared: SharedExpert | None = None,
                 act_mode: int = _lib.ACT_MODE_CANDLE, placement=None):
        """placement: None (rank r owns experts r*epr .. (r+1)*epr - 1), or the slot of every expert
        (a permutation of 0 .. n_experts-1: expert e lives on rank slot // epr at local index
        slot % epr; this rank's banks and expert biases then hold its experts in slot order, see
        expert_lists)."""
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
        self.placement = None
        if placement is not None:
            p = np.asarray(placement.cpu() if isinstance(placement, torch.Tensor) else placement, dtype=np.int64)
            if p.shape != (self.n_experts,) or not np.array_equal(np.sort(p), np.arange(self.n_experts)):
                raise ValueError("placement must be a permutation of the expert indices")
            self.placement = torch.from_numpy(p.astype(np.int32)).to(self.gate.device)
        self._group = _lib.EpGroup(world, rank, self.epr, _ptr(self.placement))
        self.row_dtype = torch.float16 if _lib.lib().cwx_ep_rows_f16(ctypes.byref(L)) else torch.float32

    def dispatch(self, x: torch.Tensor) -> Dispatched:
        T, H = x.shape
        W = self._group.world
        n = T * self.top_k
        dev = x.device
        ids = torch.empty(n, dtype=torch.int32, device=dev)
        w = torch.empty(n, dtype=torch.float32, device=dev)
        sgate = torch.empty(T, dtype=torch.float32, device=dev) if self.shared is not None else None
        unit_of = torch.empty((T, W), dtype=torch.int32, device=dev)
        rows = torch.empty((T * min(self.top_k, W), H), dtype=self.row_dtype, device=dev)
        picks = torch.empty((n, 3), dtype=torch.int32, device=dev)
        counts = torch.empty((W, 2), dtype=torch.int32, device=dev)
        check(_lib.lib().cwx_ep_dispatch(_lib.ctx(_dev_index(x)), ctypes.byref(self._layer), ctypes.byref(self._group),
                                         x.data_ptr(), T, ids.data_ptr(), w.data_ptr(), _ptr(sgate),
                                         unit_of.data_ptr(), rows.data_ptr(), picks.data_ptr(), counts.data_ptr(),
                                         _stream(dev)))
        return Dispatched(x, ids.view(T, self.top_k), unit_of, sgate, rows, picks, counts)

    def experts(self, rows: torch.Tensor, picks: torch.Tensor, src_units: list[int],
                src_picks: list[int]) -> torch.Tensor:
        nu, npk = rows.shape[0], picks.shape[0]
        y = torch.empty((nu, self.hidden), dtype=torch.float32, device=rows.device)
        if npk:
            su = (ctypes.c_int32 * len(src_units))(*src_units)
            sp = (ctypes.c_int32 * len(src_picks))(*src_picks)
            check(_lib.lib().cwx_ep_experts(_lib.ctx(_dev_index(rows)), ctypes.byref(self._layer),
                                            ctypes.byref(self._group), rows.data_ptr(), picks.data_ptr(), nu, npk,
                                            len(src_units), su, sp, y.data_ptr(), _stream(rows.device)))
        return y

    def combine(self, d: Dispatched, back: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        T, H = d.x.shape
        out = torch.empty((T, H), dtype=torch.float32, device=d.x.device)
        check(_lib.lib().cwx_ep_combine(_lib.ctx(_dev_index(d.x)), ctypes.byref(self._layer),
                                        ctypes.byref(self._group), d.x.data_ptr(), T, d.unit_of.data_ptr(),
                                        back.data_ptr(), _ptr(d.sgate), _ptr(residual), out.data_ptr(),
                                        _stream(d.x.device)))
        return out


def balanced_placement(counts, world: int) -> np.ndarray:
    """Slots of a placement that spreads the experts' expected picks (counts, e.g. of a calibration
    batch) over `world` ranks of n_experts / world experts each: the experts in decreasing count,
    each to the least loaded rank that still has room (ties to the lowest rank), in its next
    local slot."""
    counts = np.asarray(counts, dtype=np.float64)
    E = counts.size
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    epr = E // world
    load, used = np.zeros(world), np.zeros(world, dtype=np.int64)
    slot = np.empty(E, dtype=np.int32)
    for e in np.argsort(-counts, kind="stable"):
        r = min((r for r in range(world) if used[r] < epr), key=lambda r: (load[r], r))
        slot[e] = r * epr + used[r]
        load[r] += counts[e]
        used[r] += 1
    return slot


def expert_lists(slot, world: int) -> list[list[int]]:
    """The experts of each rank in local-slot order under a placement."""
    slot = np.asarray(slot)
    epr = slot.size // world
    order = np.argsort(slot)
    return [order[r * epr:(r + 1) * epr].tolist() for r in range(world)]


class ExpertParallelMoe:
    """One MoE layer whose experts are split over the ranks of `group` (torch.distributed)."""

    def __init__(self, engine, group=None):
        import torch.distributed as dist

        self.engine, self.group = engine, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.timer = None  # optional: .mark(phase) called at the start of each phase (benchmarks)

    def _mark(self, name: str) -> None:
        if self.timer is not None:
            self.timer.mark(name)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        import torch.distributed as dist

        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, xs: torch.Tensor, residual: torch.Tensor | None = None,
                taps: dict | None = None) -> torch.Tensor:
        """xs (b, s, h) local tokens -> this rank's layer output, in the input's dtype. taps, when
        given, receives the local tokens' expert ids ("ids", (tokens, top_k))."""
        b, s, h = xs.shape
        x = xs.reshape(b * s, h).to(torch.float32).contiguous()
        res = None if residual is None else residual.reshape(b * s, h).to(torch.float32).contiguous()
        self._mark("dispatch")
        d = self.engine.dispatch(x)
        if taps is not None and d.ids is not None:
            taps["ids"] = d.ids
        self._mark("counts_exchange_and_host_read")
        # counts first: every rank learns how many units and records each peer sends it
        recv_counts = torch.empty_like(d.send_counts)
        if self.world == 1:
            recv_counts.copy_(d.send_counts)
        else:
            import torch.distributed as dist

            dist.all_to_all_single(recv_counts, d.send_counts, group=self.group)
        sc, rc = d.send_counts.tolist(), recv_counts.tolist()
        su, sp = [int(v[0]) for v in sc], [int(v[1]) for v in sc]
        ru, rp = [int(v[0]) for v in rc], [int(v[1]) for v in rc]
        rows = torch.empty((sum(ru), h), dtype=d.send_rows.dtype, device=x.device)
        picks = torch.empty((sum(rp), 3), dtype=torch.int32, device=x.device)
        self._mark("row_exchange")
        self._a2a(rows, d.send_rows[:sum(su)], ru, su)
        self._a2a(picks, d.send_picks[:sum(sp)], rp, sp)
        self._mark("experts")
        y = self.engine.experts(rows, picks, ru, rp)
        back = torch.empty((sum(su), h), dtype=torch.float32, device=x.device)
        self._mark("return_exchange")
        self._a2a(back, y, su, ru)
        self._mark("combine")
        out = self.engine.combine(d, back, res)
        self._mark("end")
        return out.reshape(b, s, h).to(xs.dtype)


class EpComm:
    """This rank's communicator of the library's own expert-parallel transport (cwx_ep_comm, NCCL
    bound inside libcwx.so). Rank 0 makes the unique id; it reaches the other ranks through
    `share(id_bytes) -> id_bytes` (by default a torch.distributed object broadcast); every rank then
    creates its communicator (a collective call)."""

    def __init__(self, device: int, world: int, rank: int, share=None):
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            check(_lib.lib().cwx_ep_unique_id(uid, 128))
        raw = bytes(uid.raw)
        if share is None:
            import torch.distributed as dist

            box = [raw if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            raw = box[0]
        else:
            raw = share(raw)
        uid = ctypes.create_string_buffer(raw, 128)
        h = ctypes.c_void_p()
        check(_lib.lib().cwx_ep_comm_create(device, uid, world, rank, ctypes.byref(h)))
        self.handle, self.device, self.world, self.rank = h, device, world, rank

    def close(self) -> None:
        if self.handle:
            _lib.lib().cwx_ep_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LibraryExpertParallelMoe:
    """One expert-parallel layer run by cwx_ep_forward: dispatch, both exchanges (NCCL inside the
    library, fixed per-peer sizes, counts read on the device) and the combine in one stream-ordered
    call, no host synchronisation. Every rank calls forward with at most cap_tokens local tokens."""

    def __init__(self, engine: CudaEngine, comm: EpComm, cap_tokens: int):
        self.engine, self.comm, self.cap_tokens = engine, comm, cap_tokens

    def forward(self, xs: torch.Tensor, residual: torch.Tensor | None = None,
                taps: dict | None = None) -> torch.Tensor:
        """xs (b, s, h) local tokens -> this rank's layer output, in the input's dtype. taps, when
        given, receives the local tokens' expert ids ("ids", (tokens, top_k))."""
        b, s, h = xs.shape
        n = b * s
        if n > self.cap_tokens:
            raise ValueError(f"{n} tokens above the exchange capacity of {self.cap_tokens}")
        x = xs.reshape(n, h).to(torch.float32).contiguous()
        res = None if residual is None else residual.reshape(n, h).to(torch.float32).contiguous()
        out = torch.empty((n, h), dtype=torch.float32, device=xs.device)
        ids = None
        if taps is not None:
            ids = torch.empty((n, self.engine.top_k), dtype=torch.int32, device=xs.device)
            taps["ids"] = ids
        e = self.engine
        check(_lib.lib().cwx_ep_forward(_lib.ctx(_dev_index(xs)), self.comm.handle, ctypes.byref(e._layer),
                                        ctypes.byref(e._group), x.data_ptr(), n, self.cap_tokens, _ptr(res),
                                        out.data_ptr(), _ptr(ids), _stream(xs.device)))
        return out.reshape(b, s, h).to(xs.dtype)


__all__ = ["CudaEngine", "Dispatched", "EpComm", "ExpertParallelMoe", "LibraryExpertParallelMoe"]
