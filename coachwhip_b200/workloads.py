"""The benchmark configurations as synthetic MoE layers on the device.

BASELINE's five configurations of coachwhip's MoE layer, with every tensor drawn from the
library's seeded generator (cwx_bank_synth / cwx_synth_normal: SplitMix64 counter stream and an
own Box-Muller, the same values as the CPU oracle's generator) instead of a model file:

  C0  Qwen3.6-35B-A3B-shaped block: H2048, 256 experts, top-8 renormalised, I512, Q4_K experts
      (seed 0), one Q4_K shared expert with a sigmoid gate; x 64 x 2048 (seed 1)
  C1  the decode stack: 40 layers of the C0 shape, gate/up IQ2_S, down IQ3_S (seed 2), Q4_K shared
  C2  prefill on the C1 weights: x 1500 or 4096 tokens (seed 3)
  C3  gpt-oss-120b-shaped: H2880, 128 experts, top-4 renormalised, I2880, MXFP4 experts with
      per-expert biases, clamped SwiGLU (1.702, 7.0), router bias, no shared expert; 36 layers (seed 4)
  C4  Qwen3-Coder-Next-shaped: H2048, 512 experts, top-10, I512, gate/up IQ3_S, down Q4_K, Q4_K
      shared expert, router logits plus a Zipf(1.1) bias over a seeded permutation; 48 layers (seed 5)

Tensor t of layer l of a configuration with seed s comes from stream cwx_stream(s, l, t); the
tensor indices are the T_* constants below. The shapes follow the model families' MoE layers:
crates/engine/src/model_next.rs:1036-1053 (Qwen3-Next / Qwen3.5-MoE), model_gptoss.rs:115-197.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .moe import Bank, ExpertAct, ExpertStore, SharedExpert, StreamedMoe

T_GATE, T_UP, T_DOWN, T_RW, T_RB, T_SG, T_SU, T_SD, T_SGI, T_GB, T_UB, T_DB, T_IN = range(13)


@dataclass(frozen=True)
class Config:
    name: str
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    gate_type: int
    up_type: int
    down_type: int
    layers: int
    seed: int
    input_seed: int
    shared_inter: int = 0
    sh_type: int = _lib.TYPE_Q4_K
    act: int = _lib.ACT_SILU
    router_bias: bool = False
    expert_bias: bool = False
    zipf: float = 0.0
    w_std: float = 0.02

    def expert_bytes(self) -> int:
        """Quantised bytes of one routed expert (gate + up + down)."""
        from .moe import row_bytes

        return (row_bytes(self.gate_type, self.hidden) * self.inter + row_bytes(self.up_type, self.hidden) * self.inter
                + row_bytes(self.down_type, self.inter) * self.hidden)

    def shared_bytes(self) -> int:
        from .moe import row_bytes

        if not self.shared_inter:
            return 0
        return 2 * row_bytes(self.sh_type, self.hidden) * self.shared_inter + row_bytes(self.sh_type,
                                                                                          self.shared_inter) * self.hidden

    def flops(self, T: int) -> int:
        """Algorithmic multiply-add FLOPs of one layer on T tokens: routed gate/up/down, shared
        expert, router."""
        return (2 * T * self.top_k * 3 * self.hidden * self.inter + 2 * T * 3 * self.hidden * self.shared_inter
                + 2 * T * self.hidden * self.n_experts)


Q4K, IQ2S, IQ3S, MXFP4 = _lib.TYPE_Q4_K, _lib.TYPE_IQ2_S, _lib.TYPE_IQ3_S, _lib.TYPE_MXFP4
CONFIGS = {
    "C0": Config("C0", 2048, 256, 8, 512, Q4K, Q4K, Q4K, 1, seed=0, input_seed=1, shared_inter=512),
    "C1": Config("C1", 2048, 256, 8, 512, IQ2S, IQ2S, IQ3S, 40, seed=2, input_seed=2, shared_inter=512),
    "C2": Config("C2", 2048, 256, 8, 512, IQ2S, IQ2S, IQ3S, 40, seed=2, input_seed=3, shared_inter=512),
    "C3": Config("C3", 2880, 128, 4, 2880, MXFP4, MXFP4, MXFP4, 36, seed=4, input_seed=5,
                 act=_lib.ACT_CLAMPED_SWIGLU, router_bias=True, expert_bias=True),
    "C4": Config("C4", 2048, 512, 10, 512, IQ3S, IQ3S, Q4K, 48, seed=5, input_seed=6, shared_inter=512, zipf=1.1),
}


def stream(seed: int, layer: int, tensor: int) -> int:
    """cwx_stream(): the per-tensor key of the seeded generator."""

    def sm(x):
        x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return x ^ (x >> 31)

    return sm((seed << 40) ^ (layer << 16) ^ tensor)


def normal(n: int, key: int, std: float, device: int, offset: int = 0) -> torch.Tensor:
    """n N(0, std^2) f32 values of stream `key` on the device."""
    out = torch.empty(n, dtype=torch.float32, device=f"cuda:{device}")
    _lib.check(_lib.lib().cwx_synth_normal(_lib.ctx(device), key, offset, n, std, out.data_ptr(),
                                           torch.cuda.current_stream(device).cuda_stream))
    return out


def zipf_bias(cfg: Config) -> np.ndarray:
    """ln of the Zipf(s) pmf at each expert's rank, the ranks a seeded permutation of 1..E."""
    E = cfg.n_experts
    r = np.random.default_rng(cfg.seed).permutation(E) + 1
    norm = np.log(np.sum(np.arange(1, E + 1, dtype=np.float64) ** -cfg.zipf))
    return (-cfg.zipf * np.log(r) - norm).astype(np.float32)


@dataclass
class Layer:
    """One synthetic layer on the device: its banks, dense tensors and the StreamedMoe over them.
    With first / n_local set, the banks and expert biases hold experts first .. first+n_local-1
    (an expert-parallel rank's slice) and `moe` is None."""

    cfg: Config
    index: int
    banks: tuple
    router_w: torch.Tensor
    router_b: torch.Tensor | None
    act: object
    shared: SharedExpert | None
    moe: StreamedMoe | None
    first: int = 0


def router(cfg: Config, layer: int, device: int = 0):
    """The layer's router weight (E, H) and bias (E, or None: the router bias, plus the Zipf bias)."""
    E, H = cfg.n_experts, cfg.hidden
    st = lambda t: stream(cfg.seed, layer, t)  # noqa: E731
    w = normal(E * H, st(T_RW), cfg.w_std, device).view(E, H)
    b = None
    if cfg.router_bias:
        b = normal(E, st(T_RB), cfg.w_std, device)
    if cfg.zipf:
        z = torch.from_numpy(zipf_bias(cfg)).to(f"cuda:{device}")
        b = z if b is None else b + z
    return w, b


def build_layer(cfg: Config, layer: int, device: int = 0, act_mode: int = _lib.ACT_MODE_CANDLE,
                first: int = 0, n_local: int | None = None, store: ExpertStore | None = None,
                experts=None) -> Layer:
    """Layer `layer` of configuration cfg, synthesised on `device`. `experts` (a list of global
    expert indices) makes an expert-parallel rank's layer under a placement: its banks and expert
    biases hold those experts in list order."""
    E, H, I = cfg.n_experts, cfg.hidden, cfg.inter
    st = lambda t: stream(cfg.seed, layer, t)  # noqa: E731
    if experts is not None:
        experts = [int(e) for e in experts]
        n_local = len(experts)
        g = Bank.synth_list(cfg.gate_type, I, H, experts, st(T_GATE), cfg.w_std, device)
        u = Bank.synth_list(cfg.up_type, I, H, experts, st(T_UP), cfg.w_std, device)
        d = Bank.synth_list(cfg.down_type, H, I, experts, st(T_DOWN), cfg.w_std, device)
    else:
        ne = E if n_local is None else n_local
        g = Bank.synth(cfg.gate_type, I, H, ne, st(T_GATE), cfg.w_std, device, first=first)
        u = Bank.synth(cfg.up_type, I, H, ne, st(T_UP), cfg.w_std, device, first=first)
        d = Bank.synth(cfg.down_type, H, I, ne, st(T_DOWN), cfg.w_std, device, first=first)
    ne = E if n_local is None else n_local
    w, b = router(cfg, layer, device)
    if cfg.act == _lib.ACT_CLAMPED_SWIGLU:
        rows = (slice(first, first + ne) if experts is None
                else torch.tensor(experts, dtype=torch.long, device=f"cuda:{device}"))
        bias = lambda t, n: (normal(E * n, st(t), cfg.w_std, device).view(E, n)[rows].contiguous()  # noqa
                             if cfg.expert_bias else None)
        act = ExpertAct.ClampedSwiglu(1.702, 7.0, bias(T_GB, I), bias(T_UB, I), bias(T_DB, H))
    else:
        act = ExpertAct.Silu()
    shared = None
    if cfg.shared_inter:
        Is = cfg.shared_inter
        shared = SharedExpert(normal(H, st(T_SGI), cfg.w_std, device),
                              Bank.synth(cfg.sh_type, Is, H, 1, st(T_SG), cfg.w_std, device),
                              Bank.synth(cfg.sh_type, Is, H, 1, st(T_SU), cfg.w_std, device),
                              Bank.synth(cfg.sh_type, H, Is, 1, st(T_SD), cfg.w_std, device))
    moe = None
    if n_local is None:
        if store is None:
            store = ExpertStore([(g, u, d)])
            li = 0
        else:
            store.banks.append((g, u, d))
            li = len(store.banks) - 1
        moe = StreamedMoe(li, w, cfg.top_k, True, act, store, gate_bias=b, shared=shared, act_mode=act_mode)
    return Layer(cfg, layer, (g, u, d), w, b, act, shared, moe, first)


def make_input(cfg: Config, T: int, device: int = 0, layer: int = 0) -> torch.Tensor:
    """x (T, hidden) f32 N(0, 1): the configuration's input seed."""
    return normal(T * cfg.hidden, stream(cfg.input_seed, layer, T_IN), 1.0, device).view(T, cfg.hidden)


def oracle_layer(lay: Layer) -> dict:
    """The layer's bytes and tensors on the host, under the CPU oracle's field names."""
    cfg = lay.cfg
    g, u, d = lay.banks
    t = lambda x: None if x is None else x.detach().cpu().numpy()  # noqa: E731
    L = dict(hidden=cfg.hidden, n_experts=cfg.n_experts, top_k=cfg.top_k, inter=cfg.inter, norm_topk_prob=1,
             gate_type=cfg.gate_type, up_type=cfg.up_type, down_type=cfg.down_type, act=cfg.act, alpha=1.702,
             limit=7.0, gate_bank=g.download(), up_bank=u.download(), down_bank=d.download(),
             router_w=t(lay.router_w))
    if lay.router_b is not None:
        L["router_b"] = t(lay.router_b)
    if isinstance(lay.act, ExpertAct.ClampedSwiglu):
        for k in ("gate_b", "up_b", "down_b"):
            if getattr(lay.act, k) is not None:
                L[k] = t(getattr(lay.act, k))
    if lay.shared is not None:
        s = lay.shared
        L.update(shared_inter=cfg.shared_inter, sh_gate_type=cfg.sh_type, sh_up_type=cfg.sh_type,
                 sh_down_type=cfg.sh_type, sh_gate=s.gate.download(), sh_up=s.up.download(),
                 sh_down=s.down.download(), sh_gate_inp=t(s.gate_inp))
    return L
