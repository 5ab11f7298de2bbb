"""Tensor-core (tcgen05) expert products of large piles against the CPU oracle.

Layers whose routed banks are codebook IQ formats (IQ2_S, IQ3_S, IQ2_XXS, IQ3_XXS), Q4_K under the
f32 policy, or MXFP4 with every block scale in the f16-exact range take these products once the
batch gives enough picks per expert; here the threshold is dropped to 1 so every case below takes
them. Same bar as the
grouped mma.sync products: MoE output within relative L2 1e-3 of the oracle with the same
activation semantics, expert ids and piles bit-exact.
"""

import numpy as np
import pytest

import oracle as O
from tests.layers import Spec, build_cpu, build_gpu, make_input, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-3
DEV = "cuda:0"

SPECS = {
    # config-1 mix, narrow: IQ2_S gate/up (fused), IQ3_S down, Q4_K shared expert
    "iq_mix": Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_S, up_type=O.IQ2_S,
                   down_type=O.IQ3_S, shared_inter=256, seed=2),
    # IQ3_S gate/up, IQ2_S down, no shared expert
    "iq3_iq2": Spec(hidden=512, n_experts=16, top_k=4, inter=512, gate_type=O.IQ3_S, up_type=O.IQ3_S,
                    down_type=O.IQ2_S, seed=6),
    # config-1 widths (eight 256-column pieces per gate/up row), few experts: piles above 256
    # picks take several column tiles
    "iq_wide": Spec(hidden=2048, n_experts=16, top_k=2, inter=512, gate_type=O.IQ2_S, up_type=O.IQ2_S,
                    down_type=O.IQ3_S, shared_inter=512, seed=2),
    # config-4 family: IQ3_S gate/up, Q4_K down (tensor cores under the f32 policy only)
    "iq3_q4k": Spec(hidden=512, n_experts=64, top_k=10, inter=256, gate_type=O.IQ3_S, up_type=O.IQ3_S,
                    down_type=O.Q4_K, shared_inter=256, seed=5),
    # the reference file's formats: IQ2_XXS gate/up, IQ3_XXS down; IQ4_XS shared expert (grouped
    # mma.sync products beside the tensor-core ones)
    "iq_xxs": Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_XXS, up_type=O.IQ2_XXS,
                   down_type=O.IQ3_XXS, shared_inter=256, sh_types=(O.IQ4_XS, O.IQ4_XS, O.IQ4_XS), seed=8),
    # gpt-oss family (config 3): MXFP4 gate/up/down with expert biases and the clamped SwiGLU,
    # router bias; hidden and inter of 2 whole pieces and a 64-column tail piece (row-major), and
    # down rows ending with half a 128-row tile
    "mxfp4_gptoss": Spec(hidden=576, n_experts=16, top_k=4, inter=576, gate_type=O.MXFP4, up_type=O.MXFP4,
                         down_type=O.MXFP4, act=O.ACT_CLAMPED_SWIGLU, router_bias=True, expert_bias=True, seed=4),
    # IQ3_XXS gate/up, IQ2_XXS down, shared expert of the same formats on the tensor cores
    "iq3xxs_iq2xxs": Spec(hidden=768, n_experts=16, top_k=4, inter=512, gate_type=O.IQ3_XXS, up_type=O.IQ3_XXS,
                          down_type=O.IQ2_XXS, shared_inter=512, sh_types=(O.IQ3_XXS, O.IQ3_XXS, O.IQ2_XXS),
                          seed=10),
}


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.fixture(scope="module", autouse=True)
def _force_mma():
    from coachwhip_b200 import _lib

    _lib.lib()
    _lib.set_mma_min_pile(0, 1)
    yield
    _lib.status(0)
    _lib.set_mma_min_pile(0, 32)


def _launches():
    from coachwhip_b200 import _lib

    return _lib.lib().cwx_ctx_launches(_lib.ctx(0))


@pytest.mark.parametrize("name,T", [("iq_mix", 256), ("iq_mix", 1500), ("iq3_iq2", 700), ("iq_wide", 1500),
                                    ("iq3_q4k", 512), ("iq_xxs", 300), ("iq_xxs", 1500), ("iq3xxs_iq2xxs", 900),
                                    ("mxfp4_gptoss", 64), ("mxfp4_gptoss", 1200)])
@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
def test_mma_forward_matches_oracle(name, T, mode):
    from coachwhip_b200 import _lib

    s = SPECS[name]
    L = build_cpu(s)
    x = make_input(s, T)
    ref = O.moe_forward(L, x, mode)
    moe = build_gpu(L, act_mode=mode)
    taps = {}
    out = moe.forward(_t(x)[None], taps=taps)[0].cpu().numpy()
    _lib.status(0)
    assert np.array_equal(taps["ids"].cpu().numpy().astype(np.uint32), ref["ids"]), "expert ids"
    op, oh = O.permute(ref["ids"], s.n_experts)
    assert np.array_equal(taps["pairs"].cpu().numpy().view(np.uint32), op)
    err = rel_l2(out, ref["out"])
    assert err < RTOL, err


@pytest.mark.parametrize("name", ["iq_mix", "mxfp4_gptoss"])
def test_mma_path_is_taken_and_matches_mma_sync(name):
    """Same layer and batch through both product paths: different launch sequences, outputs
    within the bar of each other."""
    from coachwhip_b200 import _lib

    s = SPECS[name]
    L = build_cpu(s)
    x = _t(make_input(s, 512))[None]
    moe = build_gpu(L)
    outs, launches = [], []
    for pile in (1, 0):
        _lib.set_mma_min_pile(0, pile)
        moe.forward(x)  # workspace sized outside the count
        torch.cuda.synchronize()
        n0 = _launches()
        outs.append(moe.forward(x).cpu().numpy())
        launches.append(_launches() - n0)
    _lib.set_mma_min_pile(0, 1)
    _lib.status(0)
    assert launches[0] != launches[1], launches
    assert rel_l2(outs[0], outs[1]) < RTOL


def test_mma_skewed_piles():
    # two experts take every token: piles of T picks, several column tiles each
    from coachwhip_b200 import _lib

    s = Spec(hidden=512, n_experts=16, top_k=2, inter=256, gate_type=O.IQ2_S, up_type=O.IQ2_S,
             down_type=O.IQ3_S, seed=7)
    L = build_cpu(s)
    L["router_b"] = np.zeros(16, dtype=np.float32)
    L["router_b"][3] = 50.0
    L["router_b"][9] = 49.0
    x = make_input(s, 600)
    ref = O.moe_forward(L, x, O.MODE_F32)
    moe = build_gpu(L, act_mode=O.MODE_F32)
    out = moe.forward(_t(x)[None])[0].cpu().numpy()
    _lib.status(0)
    assert rel_l2(out, ref["out"]) < RTOL


def test_mxfp4_outside_the_f16_range_stays_on_mma_sync():
    # block scales far below 2^-24 (weights near 1e-12): code * 2^(e - 128) is not exact in f16,
    # so the bank is not marked for the tensor cores and the layer keeps the grouped products
    from coachwhip_b200 import _lib

    s = Spec(hidden=512, n_experts=8, top_k=2, inter=256, gate_type=O.MXFP4, up_type=O.MXFP4,
             down_type=O.MXFP4, act=O.ACT_CLAMPED_SWIGLU, expert_bias=True, seed=11, w_std=1e-12)
    L = build_cpu(s)
    x = _t(make_input(s, 512))[None]
    moe = build_gpu(L)
    launches = []
    for pile in (1, 0):
        _lib.set_mma_min_pile(0, pile)
        moe.forward(x)
        torch.cuda.synchronize()
        n0 = _launches()
        moe.forward(x)
        launches.append(_launches() - n0)
    _lib.set_mma_min_pile(0, 1)
    _lib.status(0)
    assert launches[0] == launches[1], launches
