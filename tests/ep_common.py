"""Shared pieces of the expert-parallel tests: a CPU engine built on the oracle (test
infrastructure only) and the per-rank GPU engine over banks sliced from the oracle's bytes."""

from __future__ import annotations

import numpy as np

import oracle as O


def expert_bytes(L: dict, which: str) -> int:
    H, I = L["hidden"], L["inter"]
    t = L[f"{which}_type"]
    n, k = (I, H) if which in ("gate", "up") else (H, I)
    return n * O.row_bytes(t, k)


class OracleEngine:
    """This rank's steps on the CPU with the oracle's primitives (router, route, per-expert
    products, layer forward for the shared expert), on the same unit protocol as CudaEngine."""

    def __init__(self, L: dict, world: int, rank: int, mode: int):
        self.L, self.world, self.rank, self.mode = L, world, rank, mode
        self.E, self.K, self.H, self.I = L["n_experts"], L["top_k"], L["hidden"], L["inter"]
        self.epr = self.E // world

    def dispatch(self, x):
        import torch

        from coachwhip_b200.ep import Dispatched

        L, K, W = self.L, self.K, self.world
        xn = x.numpy()
        T = xn.shape[0]
        logits = O.router(xn, L["router_w"], L.get("router_b"))
        ids, w = O.route(logits, K, bool(L["norm_topk_prob"]))
        unit_of = -np.ones((T, W), dtype=np.int32)
        rows, recs, counts = [], [], np.zeros((W, 2), dtype=np.int32)
        for d in range(W):  # destinations in rank order, their units in token order
            for t in range(T):
                js = [j for j in range(K) if ids[t, j] // self.epr == d]
                if not js:
                    continue
                u = counts[d, 0]
                unit_of[t, d] = len(rows)
                rows.append(xn[t])
                for j in js:
                    recs.append((u, ids[t, j] % self.epr, np.float32(w[t, j]).view(np.int32)))
                counts[d, 0] += 1
                counts[d, 1] += len(js)
        rows = np.array(rows, dtype=np.float32).reshape(-1, self.H)
        recs = np.array(recs, dtype=np.int32).reshape(-1, 3)
        return Dispatched(x, torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(unit_of), None,
                          torch.from_numpy(rows), torch.from_numpy(recs), torch.from_numpy(counts))

    def experts(self, rows, picks, src_units, src_picks):
        import torch

        L, H, I = self.L, self.H, self.I
        r, pk = rows.numpy(), picks.numpy()
        uoff = np.concatenate([[0], np.cumsum(src_units)])
        poff = np.concatenate([[0], np.cumsum(src_picks)])
        unit = np.concatenate([pk[poff[s]:poff[s + 1], 0] + uoff[s] for s in range(len(src_units))]).astype(np.int64)
        eid, wgt = pk[:, 1], pk[:, 2].view(np.float32)
        y = np.zeros((pk.shape[0], H), dtype=np.float32)
        for el in np.unique(eid):
            sel = np.nonzero(eid == el)[0]
            e = int(self.rank * self.epr + el)
            xr = r[unit[sel]]
            g = O.matmul(L["gate_type"], self.mode, L["gate_bank"], I, H, expert_bytes(L, "gate"), e, xr)
            u = O.matmul(L["up_type"], self.mode, L["up_bank"], I, H, expert_bytes(L, "up"), e, xr)
            if L.get("act", O.ACT_SILU) == O.ACT_CLAMPED_SWIGLU:
                # gpt-oss: biases of expert e, gate clamped above, up clamped both ways
                lim, alpha = np.float32(L.get("limit", 7.0)), np.float32(L.get("alpha", 1.702))
                if L.get("gate_b") is not None:
                    g = g + L["gate_b"][e]
                if L.get("up_b") is not None:
                    u = u + L["up_b"][e]
                g = np.minimum(g, lim)
                u = np.clip(u, -lim, lim)
                h = (u + np.float32(1)) * (g / (np.exp(-g * alpha) + np.float32(1)))
            else:
                h = (g / (np.float32(1) + np.exp(-g))) * u
            y[sel] = O.matmul(L["down_type"], self.mode, L["down_bank"], H, I, expert_bytes(L, "down"), e,
                              h.astype(np.float32))
            if L.get("act", O.ACT_SILU) == O.ACT_CLAMPED_SWIGLU and L.get("down_b") is not None:
                y[sel] = y[sel] + L["down_b"][e]
        yu = np.zeros((r.shape[0], H), dtype=np.float32)
        for p in range(pk.shape[0]):  # each unit's weighted sum in record order
            yu[unit[p]] += wgt[p] * y[p]
        return torch.from_numpy(yu)

    def combine(self, d, back, residual):
        import torch

        b = back.numpy()
        uo = d.unit_of.numpy()
        T = uo.shape[0]
        out = np.zeros((T, self.H), dtype=np.float32)
        for dd in range(self.world):
            has = uo[:, dd] >= 0
            out[has] += b[uo[has, dd]]
        out += O.moe_forward(self.L, d.x.numpy(), self.mode)["shared"]
        if residual is not None:
            out += residual.numpy()
        return torch.from_numpy(out)


def gpu_engine(L: dict, world: int, rank: int, device: int, act_mode: int, placement=None):
    """CudaEngine for rank `rank`: banks of its experts (and their bias rows) from the oracle's bytes;
    with a placement (every expert's slot), the experts it assigns to this rank in slot order."""
    import torch

    from coachwhip_b200.ep import CudaEngine, expert_lists
    from coachwhip_b200.moe import Bank, ExpertAct, SharedExpert

    dev = f"cuda:{device}"
    H, E, I = L["hidden"], L["n_experts"], L["inter"]
    epr = E // world
    mine = list(range(rank * epr, (rank + 1) * epr)) if placement is None else expert_lists(placement, world)[rank]

    def sl(name):
        b = expert_bytes(L, name)
        return np.concatenate([L[f"{name}_bank"][e * b:(e + 1) * b] for e in mine])

    g = Bank.from_gguf_bytes(sl("gate"), L["gate_type"], I, H, epr, device)
    u = Bank.from_gguf_bytes(sl("up"), L["up_type"], I, H, epr, device)
    dn = Bank.from_gguf_bytes(sl("down"), L["down_type"], H, I, epr, device)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)  # noqa
    if L.get("act", 0) == 1:
        rows = lambda a: None if a is None else a[mine]  # noqa: E731
        act = ExpertAct.ClampedSwiglu(L.get("alpha", 1.702), L.get("limit", 7.0), t(rows(L.get("gate_b"))),
                                      t(rows(L.get("up_b"))), t(rows(L.get("down_b"))))
    else:
        act = ExpertAct.Silu()
    shared = None
    if L.get("shared_inter"):
        Is = L["shared_inter"]
        shared = SharedExpert(t(L["sh_gate_inp"]),
                              Bank.from_gguf_bytes(L["sh_gate"], L["sh_gate_type"], Is, H, 1, device),
                              Bank.from_gguf_bytes(L["sh_up"], L["sh_up_type"], Is, H, 1, device),
                              Bank.from_gguf_bytes(L["sh_down"], L["sh_down_type"], H, Is, 1, device))
    eng = CudaEngine(t(L["router_w"]), L["top_k"], bool(L["norm_topk_prob"]), act, (g, u, dn), world, rank,
                     gate_bias=t(L.get("router_b")), shared=shared, act_mode=act_mode, placement=placement)
    eng._keep = (act, shared, g, u, dn)
    return eng


def run_emulated(engines, x):
    """All ranks' engines stepped on device 0, the exchanges done by slicing: x (T, H) split
    evenly over the ranks; returns the concatenated outputs."""
    import torch

    world = len(engines)
    T = x.shape[0]
    per = T // world
    xs = [torch.from_numpy(np.ascontiguousarray(x[r * per:(r + 1) * per])).cuda() for r in range(world)]
    ds = [engines[r].dispatch(xs[r]) for r in range(world)]
    counts = [d.send_counts.cpu().numpy() for d in ds]  # (world, 2): units, records per destination
    uo = [np.concatenate([[0], np.cumsum(c[:, 0])]) for c in counts]
    po = [np.concatenate([[0], np.cumsum(c[:, 1])]) for c in counts]
    ys = []
    for dst in range(world):  # units and records for rank dst, from every source in rank order
        rows = torch.cat([ds[s].send_rows[uo[s][dst]:uo[s][dst + 1]] for s in range(world)])
        picks = torch.cat([ds[s].send_picks[po[s][dst]:po[s][dst + 1]] for s in range(world)])
        su = [int(counts[s][dst, 0]) for s in range(world)]
        sp = [int(counts[s][dst, 1]) for s in range(world)]
        ys.append((engines[dst].experts(rows, picks, su, sp), su))
    outs = []
    for s in range(world):  # unit rows back to each source, in the order it sent them
        parts = []
        for dst in range(world):
            y, su = ys[dst]
            o = int(np.sum(su[:s]))
            parts.append(y[o:o + su[s]])
        outs.append(engines[s].combine(ds[s], torch.cat(parts), None))
    from coachwhip_b200 import _lib

    _lib.status(0)
    return np.concatenate([o.cpu().numpy() for o in outs])
