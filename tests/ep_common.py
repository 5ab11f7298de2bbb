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
    """This rank's steps on the CPU with the oracle's primitives (router, route, piles, per-expert
    products, layer forward for the shared expert)."""

    def __init__(self, L: dict, world: int, rank: int, mode: int):
        self.L, self.world, self.rank, self.mode = L, world, rank, mode
        self.E, self.K, self.H, self.I = L["n_experts"], L["top_k"], L["hidden"], L["inter"]
        self.epr = self.E // world

    def dispatch(self, x):
        import torch

        from coachwhip_b200.ep import Dispatched

        L, K = self.L, self.K
        xn = x.numpy()
        logits = O.router(xn, L["router_w"], L.get("router_b"))
        ids, w = O.route(logits, K, bool(L["norm_topk_prob"]))
        pairs, _ = O.permute(ids, self.E)
        e = ids.reshape(-1)[pairs]
        rows = np.ascontiguousarray(xn[pairs // K])
        counts = np.bincount(e // self.epr, minlength=self.world).astype(np.int32)
        return Dispatched(x, torch.from_numpy(w), torch.from_numpy(pairs.astype(np.int32)), None,
                          torch.from_numpy(rows), torch.from_numpy((e % self.epr).astype(np.int32)),
                          torch.from_numpy(counts))

    def experts(self, rows, eids):
        import torch

        L, H, I = self.L, self.H, self.I
        r, ei = rows.numpy(), eids.numpy()
        y = np.zeros((r.shape[0], H), dtype=np.float32)
        for el in np.unique(ei):
            sel = np.nonzero(ei == el)[0]
            e = int(self.rank * self.epr + el)
            g = O.matmul(L["gate_type"], self.mode, L["gate_bank"], I, H, expert_bytes(L, "gate"), e, r[sel])
            u = O.matmul(L["up_type"], self.mode, L["up_bank"], I, H, expert_bytes(L, "up"), e, r[sel])
            h = (g / (np.float32(1) + np.exp(-g))) * u
            y[sel] = O.matmul(L["down_type"], self.mode, L["down_bank"], H, I, expert_bytes(L, "down"), e,
                              h.astype(np.float32))
        return torch.from_numpy(y)

    def combine(self, d, back, residual):
        import torch

        K = self.K
        pairs = d.pairs.numpy().astype(np.int64)
        inv = np.empty_like(pairs)
        inv[pairs] = np.arange(pairs.size)
        b = back.numpy()
        w = d.weights.numpy()
        T = w.shape[0]
        out = np.zeros((T, self.H), dtype=np.float32)
        for j in range(K):
            out += w[:, j:j + 1] * b[inv[np.arange(T) * K + j]]
        out += O.moe_forward(self.L, d.x.numpy(), self.mode)["shared"]
        if residual is not None:
            out += residual.numpy()
        return torch.from_numpy(out)


def gpu_engine(L: dict, world: int, rank: int, device: int, act_mode: int):
    """CudaEngine for rank `rank`: banks of its experts (and their bias rows) from the oracle's bytes."""
    import torch

    from coachwhip_b200.ep import CudaEngine
    from coachwhip_b200.moe import Bank, ExpertAct, SharedExpert

    dev = f"cuda:{device}"
    H, E, I = L["hidden"], L["n_experts"], L["inter"]
    epr = E // world
    e0, e1 = rank * epr, (rank + 1) * epr
    sl = lambda name: L[f"{name}_bank"][e0 * expert_bytes(L, name):e1 * expert_bytes(L, name)]  # noqa: E731
    g = Bank.from_gguf_bytes(sl("gate"), L["gate_type"], I, H, epr, device)
    u = Bank.from_gguf_bytes(sl("up"), L["up_type"], I, H, epr, device)
    dn = Bank.from_gguf_bytes(sl("down"), L["down_type"], H, I, epr, device)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)  # noqa
    if L.get("act", 0) == 1:
        rows = lambda a: None if a is None else a[e0:e1]  # noqa: E731
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
                     gate_bias=t(L.get("router_b")), shared=shared, act_mode=act_mode)
    eng._keep = (act, shared, g, u, dn)
    return eng
