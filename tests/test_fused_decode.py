"""The fused decode layer (one cooperative launch per layer for batches of up to 4 tokens) against
the general path and the CPU oracle.

Same routing (expert ids, routing weights and piles identical to the general path's and the
oracle's), outputs within relative L2 1e-3 of the oracle and 1e-5 of the general path (the same
products, summed in a different piece order), deterministic."""

import numpy as np
import pytest

import oracle as O
from tests.layers import Spec, build_cpu, build_gpu, make_input, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"
SPECS = {
    # config-1 formats and widths: IQ2_S gate/up, IQ3_S down, Q4_K shared expert
    "c1_shape": Spec(hidden=2048, n_experts=64, top_k=8, inter=512, gate_type=O.IQ2_S, up_type=O.IQ2_S,
                     down_type=O.IQ3_S, shared_inter=512, seed=2),
    # no shared expert, IQ3_S gate/up with IQ2_S down, 10 picks, narrow hidden
    "iq3_iq2": Spec(hidden=512, n_experts=48, top_k=6, inter=256, gate_type=O.IQ3_S, up_type=O.IQ3_S,
                    down_type=O.IQ2_S, seed=6),
    # the reference file's formats (IQ2_XXS / IQ3_XXS), Q4_K shared expert, unnormalised weights
    "xxs": Spec(hidden=1024, n_experts=32, top_k=4, inter=768, gate_type=O.IQ2_XXS, up_type=O.IQ2_XXS,
                down_type=O.IQ3_XXS, shared_inter=256, seed=8, norm=False),
}


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _launches():
    from coachwhip_b200 import _lib

    return _lib.lib().cwx_ctx_launches(_lib.ctx(0))


@pytest.fixture(scope="module", autouse=True)
def _lib_state():
    from coachwhip_b200 import _lib

    _lib.lib()
    yield
    _lib.set_fused_decode(0, 4)
    _lib.status(0)


@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("T", [1, 2, 4])
@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
def test_fused_matches_general_path_and_oracle(name, T, mode):
    from coachwhip_b200 import _lib

    s = SPECS[name]
    L = build_cpu(s)
    x = make_input(s, T)
    r = make_input(s, T, seed=77)
    moe = build_gpu(L, act_mode=mode)
    outs, taps, launches = [], [], []
    for fused in (4, 0):
        _lib.set_fused_decode(0, fused)
        tp = {}
        moe.forward(_t(x)[None], residual=_t(r)[None])  # workspace sized outside the count
        torch.cuda.synchronize()
        n0 = _launches()
        outs.append(moe.forward(_t(x)[None], residual=_t(r)[None], taps=tp)[0].cpu().numpy())
        launches.append(_launches() - n0)
        _lib.status(0)
        taps.append({k: v.cpu().numpy() for k, v in tp.items()})
    _lib.set_fused_decode(0, 4)
    assert launches[0] == 1 and launches[1] > 1, launches  # the fused path is the one launch
    for k in ("ids", "weights", "pairs", "heads"):
        assert np.array_equal(taps[0][k].view(np.uint32), taps[1][k].view(np.uint32)), k
    assert rel_l2(outs[0], outs[1]) < 1e-5
    ref = O.moe_forward(L, x, mode)
    assert np.array_equal(taps[0]["ids"].astype(np.uint32), ref["ids"])
    assert rel_l2(outs[0], ref["out"] + r) < 1e-3


def test_fused_is_deterministic_and_falls_back_above_four_tokens():
    from coachwhip_b200 import _lib

    s = SPECS["c1_shape"]
    L = build_cpu(s)
    moe = build_gpu(L)
    x = _t(make_input(s, 4))[None]
    a = moe.forward(x).cpu().numpy()
    b = moe.forward(x).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    x5 = _t(make_input(s, 5))[None]
    moe.forward(x5)
    torch.cuda.synchronize()
    n0 = _launches()
    moe.forward(x5)
    _lib.status(0)
    assert _launches() - n0 > 1  # five tokens take the general path


def test_fused_skewed_pile():
    # every token picks the same experts: piles of T picks in one expert
    from coachwhip_b200 import _lib

    s = SPECS["c1_shape"]
    L = build_cpu(s)
    L["router_b"] = np.zeros(s.n_experts, dtype=np.float32)
    L["router_b"][5] = 40.0
    L["router_b"][17] = 39.0
    x = make_input(s, 4)
    moe = build_gpu(L)
    out = moe.forward(_t(x)[None])[0].cpu().numpy()
    _lib.status(0)
    ref = O.moe_forward(L, x, O.MODE_CANDLE)
    assert rel_l2(out, ref["out"]) < 1e-3
