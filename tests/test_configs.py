"""Parity at the benchmark configurations' own shapes and seeds.

Each case synthesises layer 0 of a configuration on the GPU (the generator is pinned to the CPU
one by test_gpu_parity.py::test_synth_bank_matches_cpu_generator), runs the whole layer through
cwx_moe_forward at the configuration's batch, downloads the banks' GGUF bytes and checks against
the CPU oracle on the same bytes and inputs:
  - expert ids and the permutation (pairs, heads) bit-exact over every token;
  - routing weights within 1 ulp (bit-exact in practice) over every token;
  - the MoE output within relative L2 1e-3 of the oracle with the same activation semantics
    (CANDLE policy vs O1, F32 policy vs O2), on every token for decode batches and on an evenly
    spread sample of tokens for prefill batches. Tokens are independent in this layer (routing
    and each pick's products depend on the token's row alone), so the oracle on the sampled rows
    gives exactly the rows of the full-batch result.
The GPU runs the full batch, so the tiling, the pile sizes, the product kernel chosen (grouped
mma.sync or tcgen05) and the K-split are those of the benchmarked shapes.
"""

import numpy as np
import pytest

import oracle as O
from tests.layers import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-3
MODES = {"candle": O.MODE_CANDLE, "f32": O.MODE_F32}


@pytest.fixture(scope="module", autouse=True)
def _lib_state():
    from coachwhip_b200 import _lib

    _lib.lib()
    _lib.set_mma_min_pile(0, 32)  # the library default: prefill batches take the tensor cores
    yield
    _lib.status(0)


def _sample(T, n):
    if T <= n:
        return np.arange(T)
    return np.unique(np.linspace(0, T - 1, n).round().astype(np.int64))


def _run(name, T, mode, n_check):
    from coachwhip_b200 import _lib
    from coachwhip_b200 import workloads as W

    cfg = W.CONFIGS[name]
    lay = W.build_layer(cfg, 0, 0, act_mode=mode)
    x = W.make_input(cfg, T, 0)
    taps = {}
    out = lay.moe.forward(x[None], taps=taps)[0].cpu().numpy()
    _lib.status(0)
    L = W.oracle_layer(lay)
    xs = x.cpu().numpy()
    # routing of every token
    lg = O.router(xs, L["router_w"], L.get("router_b"))
    oi, ow = O.route(lg, cfg.top_k, True)
    gi = taps["ids"].cpu().numpy().astype(np.uint32)
    assert np.array_equal(gi, oi), f"expert ids differ on {int((gi != oi).any(1).sum())} tokens"
    ulp = np.abs(taps["weights"].cpu().numpy().view(np.int32).astype(np.int64) - ow.view(np.int32))
    assert ulp.max() <= 1, f"routing weights differ by {ulp.max()} ulp"
    op, oh = O.permute(oi, cfg.n_experts)
    assert np.array_equal(taps["pairs"].cpu().numpy().view(np.uint32), op), "permutation"
    assert np.array_equal(taps["heads"].cpu().numpy().reshape(-1).view(np.uint32), oh), "heads"
    # the layer output on the checked tokens
    rows = _sample(T, n_check)
    ref = O.moe_forward(L, xs[rows], mode)
    assert np.array_equal(ref["ids"], oi[rows])
    err = rel_l2(out[rows], ref["out"])
    assert err < RTOL, f"{name} T={T}: rel-L2 {err:.3e} over {len(rows)} tokens"
    return err


@pytest.mark.parametrize("mode", ["candle", "f32"])
def test_config0_block(mode):
    # C0: H2048, 256 Q4_K experts (seed 0), top-8, I512, Q4_K shared expert; x 64 x 2048 (seed 1)
    _run("C0", 64, MODES[mode], 64)


@pytest.mark.parametrize("T", [1, 4, 16, 64])
@pytest.mark.parametrize("mode", ["candle", "f32"])
def test_config1_decode_layer(T, mode):
    # C1: IQ2_S gate/up, IQ3_S down (seed 2), Q4_K shared; the decode batches of the benchmark
    _run("C1", T, MODES[mode], T)


@pytest.mark.parametrize("T", [1500, 4096])
@pytest.mark.parametrize("mode", ["f32", "candle"])
def test_config2_prefill_layer(T, mode):
    # C2: the C1 weights at prefill sizes (x seed 3); 47 and 128 picks per expert on average, so
    # the routed products run on the tcgen05 kernel
    _run("C2", T, MODES[mode], 256)


@pytest.mark.parametrize("T,mode,n_check", [(1, "candle", 1), (64, "candle", 64), (64, "f32", 64),
                                            (4096, "candle", 48), (4096, "f32", 96)])
def test_config3_gptoss_layer(T, mode, n_check):
    # C3: H2880, 128 MXFP4 experts with biases, top-4, I2880, clamped SwiGLU, router bias
    _run("C3", T, MODES[mode], n_check)


@pytest.mark.parametrize("mode", ["f32", "candle"])
def test_config4_zipf_layer(mode):
    # C4: 512 experts, top-10, IQ3_S gate/up, Q4_K down, Q4_K shared, Zipf(1.1) router bias;
    # 8192 tokens (the expert-parallel benchmark's whole batch) on one device
    _run("C4", 8192, MODES[mode], 192)
