"""Synthetic MoE layers built identically for the CPU oracle and the GPU library.

The quantised bytes come from the oracle's generator (bit-identical to cwx_bank_synth) and are
uploaded with cwx_bank_create, so both sides compute on the same bytes.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import oracle as O

T_GATE, T_UP, T_DOWN, T_RW, T_RB, T_SG, T_SU, T_SD, T_SGI, T_GB, T_UB, T_DB, T_IN = range(13)


@dataclass
class Spec:
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    gate_type: int
    up_type: int
    down_type: int
    seed: int = 0
    layer: int = 0
    norm: bool = True
    act: int = O.ACT_SILU
    shared_inter: int = 0
    sh_types: tuple = (O.Q4_K, O.Q4_K, O.Q4_K)
    router_bias: bool = False
    expert_bias: bool = False
    w_std: float = 0.02
    extra: dict = field(default_factory=dict)


def build_cpu(s: Spec) -> dict:
    st = lambda t: O.stream(s.seed, s.layer, t)  # noqa: E731
    E, H, I = s.n_experts, s.hidden, s.inter
    L = dict(hidden=H, n_experts=E, top_k=s.top_k, inter=I, norm_topk_prob=int(s.norm),
             gate_type=s.gate_type, up_type=s.up_type, down_type=s.down_type, act=s.act,
             alpha=1.702, limit=7.0)
    L["router_w"] = O.normal(st(T_RW), 0, E * H, s.w_std).reshape(E, H)
    if s.router_bias:
        L["router_b"] = O.normal(st(T_RB), 0, E, s.w_std)
    L["gate_bank"] = O.synth_matrix(s.gate_type, st(T_GATE), 0, E, I, H, s.w_std)
    L["up_bank"] = O.synth_matrix(s.up_type, st(T_UP), 0, E, I, H, s.w_std)
    L["down_bank"] = O.synth_matrix(s.down_type, st(T_DOWN), 0, E, H, I, s.w_std)
    if s.expert_bias:
        L["gate_b"] = O.normal(st(T_GB), 0, E * I, s.w_std).reshape(E, I)
        L["up_b"] = O.normal(st(T_UB), 0, E * I, s.w_std).reshape(E, I)
        L["down_b"] = O.normal(st(T_DB), 0, E * H, s.w_std).reshape(E, H)
    if s.shared_inter:
        Is = s.shared_inter
        L["shared_inter"] = Is
        L["sh_gate_type"], L["sh_up_type"], L["sh_down_type"] = s.sh_types
        L["sh_gate"] = O.synth_matrix(s.sh_types[0], st(T_SG), 0, 1, Is, H, s.w_std)
        L["sh_up"] = O.synth_matrix(s.sh_types[1], st(T_SU), 0, 1, Is, H, s.w_std)
        L["sh_down"] = O.synth_matrix(s.sh_types[2], st(T_SD), 0, 1, H, Is, s.w_std)
        L["sh_gate_inp"] = O.normal(st(T_SGI), 0, H, s.w_std)
    return L


def make_input(s: Spec, T: int, seed: int | None = None) -> np.ndarray:
    key = O.stream(s.seed + 1 if seed is None else seed, s.layer, T_IN)
    return O.normal(key, 0, T * s.hidden, 1.0).reshape(T, s.hidden)


def build_gpu(L: dict, device: int = 0, act_mode: int = 0):
    """StreamedMoe over banks uploaded from the oracle's bytes."""
    import torch

    from coachwhip_b200.moe import Bank, ExpertAct, ExpertStore, SharedExpert, StreamedMoe

    dev = f"cuda:{device}"
    H, E, I = L["hidden"], L["n_experts"], L["inter"]
    g = Bank.from_gguf_bytes(L["gate_bank"], L["gate_type"], I, H, E, device)
    u = Bank.from_gguf_bytes(L["up_bank"], L["up_type"], I, H, E, device)
    d = Bank.from_gguf_bytes(L["down_bank"], L["down_type"], H, I, E, device)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)  # noqa
    if L.get("act", 0) == 1:
        act = ExpertAct.ClampedSwiglu(L.get("alpha", 1.702), L.get("limit", 7.0), t(L.get("gate_b")), t(L.get("up_b")),
                                      t(L.get("down_b")))
    else:
        act = ExpertAct.Silu()
    shared = None
    if L.get("shared_inter"):
        Is = L["shared_inter"]
        shared = SharedExpert(t(L["sh_gate_inp"]),
                              Bank.from_gguf_bytes(L["sh_gate"], L["sh_gate_type"], Is, H, 1, device),
                              Bank.from_gguf_bytes(L["sh_up"], L["sh_up_type"], Is, H, 1, device),
                              Bank.from_gguf_bytes(L["sh_down"], L["sh_down_type"], H, Is, 1, device))
    moe = StreamedMoe(0, t(L["router_w"]), L["top_k"], bool(L["norm_topk_prob"]), act, ExpertStore([(g, u, d)]),
                      gate_bias=t(L.get("router_b")), shared=shared, act_mode=act_mode)
    moe._keep = (act, shared)
    return moe


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
