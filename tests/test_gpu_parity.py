"""GPU parity: libcwx.so against the CPU oracle on the same seeded inputs and bytes.

Bars: bit-exact for dequantised weights, synthetic bytes, expert ids, piles and routing weights;
MoE outputs within relative L2 1e-3 (f32 accumulate) of the oracle with the same activation
semantics (CANDLE policy vs O1, F32 policy vs O2).
"""

import numpy as np
import pytest

import oracle as O
from tests.layers import Spec, build_cpu, build_gpu, make_input, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-3  # relative L2 bound of the MoE output
FORMATS = [O.Q4_K, O.Q6_K, O.Q8_0, O.MXFP4, O.IQ2_S, O.IQ3_S, O.IQ2_XXS, O.IQ3_XXS, O.IQ4_XS]
DEV = "cuda:0"


def _t(a, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from coachwhip_b200 import _lib

    _lib.lib()
    # this module covers the grouped mma.sync products at every batch size; the tensor-core
    # products of large IQ piles have their own module (test_mma.py)
    _lib.set_mma_min_pile(0, 0)
    yield
    _lib.status(0)
    _lib.set_mma_min_pile(0, 32)


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequant_bit_exact(fmt):
    from coachwhip_b200.moe import Bank

    n, k, E = 128, 512, 3
    x = O.normal(O.stream(7, fmt, 0), 0, E * n * k, 0.02)
    x[:256] *= 40.0  # a block with large values
    x[256:512] = 0.0  # an all-zero block
    q = O.quantize(fmt, x)
    b = Bank.from_gguf_bytes(q, fmt, n, k, E)
    for e in range(E):
        got = b.dequantize(e).cpu().numpy().reshape(-1)
        want = O.dequantize(fmt, q[e * b.bytes_per_expert:(e + 1) * b.bytes_per_expert], n * k)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"expert {e}"
    assert np.array_equal(b.download(), q)


@pytest.mark.parametrize("fmt", FORMATS)
def test_synth_bank_matches_cpu_generator(fmt):
    from coachwhip_b200.moe import Bank

    n, k, E = 64, 512, 2
    key = O.stream(2, 3, 1)
    b = Bank.synth(fmt, n, k, E, key, 0.02)
    want = O.synth_matrix(fmt, key, 0, E, n, k, 0.02)
    got = b.download()
    assert np.array_equal(got, want)
    # an expert-parallel rank's slice: experts 1 .. 2 of a 3-expert tensor equal those experts
    part = Bank.synth(fmt, n, k, 2, key, 0.02, first=1).download()
    assert np.array_equal(part, O.synth_matrix(fmt, key, 1, 2, n, k, 0.02))
    # a rank's experts under a placement: a listed set, in list order
    lst = Bank.synth_list(fmt, n, k, [4, 0, 2], key, 0.02).download()
    bpe = lst.size // 3
    for i, e in enumerate([4, 0, 2]):
        assert np.array_equal(lst[i * bpe:(i + 1) * bpe], O.synth_matrix(fmt, key, e, 1, n, k, 0.02))


def test_synth_normal_matches_cpu_generator():
    import ctypes

    from coachwhip_b200 import _lib

    key = O.stream(5, 1, 12)
    n = 100_003
    out = torch.empty(n, dtype=torch.float32, device=DEV)
    _lib.check(_lib.lib().cwx_synth_normal(_lib.ctx(0), key, 17, n, 0.5, out.data_ptr(), None))
    got = out.cpu().numpy()
    want = O.normal(key, 17, n, 0.5)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


ROUTE_KATS = [  # crates/engine/tests/router.rs:21-60 and tests/lookahead.rs:6-20
    ([[0.1, 3.0, 2.0, -1.0, 1.0]], 3, True, [[1, 2, 4]]),
    ([[5.0, 0.0, 1.0, 2.0], [0.0, 1.0, 9.0, 3.0]], 2, True, [[0, 3], [2, 3]]),
    ([[0.1, 3.0, 2.0, -1.0, 1.0]], 5, False, [[1, 2, 4, 0, 3]]),
    ([[1.0, 1.0, 2.0, 1.0]], 4, False, [[2, 0, 1, 3]]),
    ([[0.5] * 6], 6, False, [[0, 1, 2, 3, 4, 5]]),
]


@pytest.mark.parametrize("case", range(len(ROUTE_KATS)))
def test_route_known_answers(case):
    from coachwhip_b200.moe import route

    logits, k, norm, want = ROUTE_KATS[case]
    lg = np.asarray(logits, dtype=np.float32)
    ids, w = route(_t(lg), k, norm)
    assert ids.cpu().numpy().tolist() == want
    oi, ow = O.route(lg, k, norm)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), oi)
    assert np.array_equal(w.cpu().numpy().view(np.uint32), ow.view(np.uint32))


@pytest.mark.parametrize("T,E,k,norm", [(64, 256, 8, True), (3, 128, 4, True), (17, 512, 10, True),
                                        (5, 96, 7, False), (1, 1000, 16, True)])
def test_route_matches_oracle(T, E, k, norm):
    from coachwhip_b200.moe import route

    lg = O.normal(O.stream(11, E, k), 0, T * E, 1.5).reshape(T, E)
    lg[0, :4] = lg[0, 4]  # exact ties
    ids, w = route(_t(lg), k, norm)
    oi, ow = O.route(lg, k, norm)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), oi)
    gw = w.cpu().numpy()
    ulp = np.abs(gw.view(np.int32).astype(np.int64) - ow.view(np.int32).astype(np.int64))
    assert ulp.max() <= 1, f"routing weights differ by {ulp.max()} ulp"
    assert (ulp == 0).mean() > 0.99


def test_rank_covers_every_expert_once():
    # crates/engine/tests/lookahead.rs:22-29: 512 scores, all ranked, in non-increasing order
    from coachwhip_b200.moe import route

    scores = np.array([((i * 7919) % 97) * 0.01 for i in range(512)], dtype=np.float32)[None, :]
    ids, _ = route(_t(scores), 16, False)
    got = ids.cpu().numpy()[0]
    assert np.all(np.diff(scores[0][got]) <= 0)
    oi, _ = O.route(scores, 16, False)
    assert np.array_equal(got.astype(np.uint32), oi[0])


def test_route_nan_does_not_fail():
    from coachwhip_b200.moe import route

    ids, _ = route(_t(np.array([[1.0, np.nan, 2.0]], dtype=np.float32)), 2, True)
    assert ids.cpu().numpy().max() < 3


# (300, 8, 12288): the largest expert count cwx_permute accepts, on the three-kernel path whose
# scan holds two words per expert in shared memory (96 KB)
@pytest.mark.parametrize("T,k,E", [(64, 8, 256), (1, 8, 256), (4096, 8, 256), (8192, 10, 512), (7, 3, 5),
                                   (300, 8, 12288), (3000, 4, 6200)])
def test_piles_match_oracle(T, k, E):
    from coachwhip_b200.moe import piles

    rng = np.random.default_rng(T + E)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    pairs, heads = piles(_t(ids.view(np.int32)), E)
    op, oh = O.permute(ids, E)
    assert np.array_equal(pairs.cpu().numpy().view(np.uint32), op)
    assert np.array_equal(heads.cpu().numpy().reshape(-1).view(np.uint32), oh)


def test_piles_bad_id_is_reported():
    from coachwhip_b200 import CwxError, _lib
    from coachwhip_b200.moe import piles

    ids = np.array([[0, 9]], dtype=np.int32)
    piles(_t(ids), 4)
    with pytest.raises(CwxError):
        _lib.status(0)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
@pytest.mark.parametrize("rpe", [False, True])
def test_expert_matmul_matches_oracle(fmt, mode, rpe):
    from coachwhip_b200.moe import Bank, MoeMatvec

    E, n, k, T, nei0 = 6, 128, 512, 9, 2
    key = O.stream(3, fmt, 2)
    q = O.synth_matrix(fmt, key, 0, E, n, k, 0.02)
    b = Bank.from_gguf_bytes(q, fmt, n, k, E)
    rng = np.random.default_rng(fmt)
    ids = np.stack([rng.permutation(E)[:nei0] for _ in range(T)]).astype(np.uint32)
    rows = T * nei0 if rpe else T
    x = O.normal(O.stream(4, fmt, 3), 0, rows * k, 1.0).reshape(rows, k)
    out = MoeMatvec(b, nei0, rpe, act_mode=mode)(_t(x), _t(ids.view(np.int32))).cpu().numpy()
    want = np.zeros_like(out)
    for t in range(T):
        for j in range(nei0):
            xr = x[t * nei0 + j] if rpe else x[t]
            want[t, j] = O.matmul(fmt, mode, q, n, k, b.bytes_per_expert, int(ids[t, j]), xr[None, :])[0]
    err = rel_l2(out, want)
    assert err < RTOL, err


@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
@pytest.mark.parametrize("spread", [20, 40])
def test_mxfp4_block_scales_far_apart(mode, spread):
    # MXFP4 block scales within a row's 256 columns: the grouped products scale each block by
    # 2^(e - max e) in f16, exact down to f16's smallest subnormal (2^-24); a bank with a piece
    # whose scales span more than 2^24 is marked when it is made and takes the exact path. Here
    # block 0 of every row has the largest e and zero codes, the row's other blocks of the first
    # piece sit 2^-spread below it (20: subnormal f16 scales on the fast path; 40: the exact
    # path), so the first piece's contribution rests on those blocks alone. Those blocks keep
    # e = 120 (weights up to 12 * 2^-8), inside the f16 range every path rounds weights to.
    from coachwhip_b200.moe import Bank, MoeMatvec

    fmt, E, n, k, T = O.MXFP4, 2, 128, 512, 5
    q = O.synth_matrix(fmt, O.stream(3, fmt, 9), 0, E, n, k, 0.02).copy()
    blocks = q.reshape(E, n, k // 32, 17)
    blocks[:, :, 0, 0] = 120 + spread
    blocks[:, :, 0, 1:] = 0
    blocks[:, :, 1:8, 0] = 120
    b = Bank.from_gguf_bytes(q, fmt, n, k, E)
    ids = np.array([[i % E] for i in range(T)], dtype=np.uint32)
    x = O.normal(O.stream(4, fmt, 9), 0, T * k, 1.0).reshape(T, k)
    out = MoeMatvec(b, 1, False, act_mode=mode)(_t(x), _t(ids.view(np.int32))).cpu().numpy()
    want = np.stack([O.matmul(fmt, mode, q, n, k, b.bytes_per_expert, int(ids[t, 0]), x[t][None, :])[0]
                     for t in range(T)])[:, None, :]
    tol = 1e-5 if mode == O.MODE_F32 else 1e-4  # (Q8_0 activation codes: the oracle's f32 block sums)
    assert rel_l2(out, want) < tol
    # the first piece alone: the second piece's blocks zeroed
    q2 = q.copy()
    q2.reshape(E, n, k // 32, 17)[:, :, 8:, 1:] = 0
    b2 = Bank.from_gguf_bytes(q2, fmt, n, k, E)
    out2 = MoeMatvec(b2, 1, False, act_mode=mode)(_t(x), _t(ids.view(np.int32))).cpu().numpy()
    want2 = np.stack([O.matmul(fmt, mode, q2, n, k, b2.bytes_per_expert, int(ids[t, 0]), x[t][None, :])[0]
                      for t in range(T)])[:, None, :]
    assert np.abs(want2).max() > 0 and rel_l2(out2, want2) < tol


def test_expert_matmul_shape_errors():
    from coachwhip_b200.moe import Bank, MoeMatvec

    q = O.synth_matrix(O.Q4_K, 1, 0, 2, 64, 256, 0.02)
    b = Bank.from_gguf_bytes(q, O.Q4_K, 64, 256, 2)
    op = MoeMatvec(b, 2, False)
    with pytest.raises(ValueError, match="ids per token"):
        op(torch.zeros((1, 256), device=DEV), torch.zeros((1, 3), dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError, match="needs contiguous"):
        op(torch.zeros((2, 512), device=DEV)[:, ::2], torch.zeros((2, 2), dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError, match="x must be f32"):
        op(torch.zeros((1, 256), device=DEV, dtype=torch.float64), torch.zeros((1, 2), dtype=torch.int32, device=DEV))


SPECS = {
    # config 0 shape family, smaller: Q4_K experts, shared expert, candle semantics
    "q4k_shared": Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.Q4_K, up_type=O.Q4_K,
                       down_type=O.Q4_K, shared_inter=256),
    # config 1 mix: IQ2_S gate/up, IQ3_S down, Q4_K shared
    "iq_mix": Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_S, up_type=O.IQ2_S,
                   down_type=O.IQ3_S, shared_inter=256, seed=2),
    # config 3 family: MXFP4, biases, clamped SwiGLU, router bias, no shared expert
    "mxfp4_gptoss": Spec(hidden=576, n_experts=16, top_k=4, inter=576, gate_type=O.MXFP4, up_type=O.MXFP4,
                         down_type=O.MXFP4, act=O.ACT_CLAMPED_SWIGLU, router_bias=True, expert_bias=True, seed=4),
    # config 4 family: IQ3_S gate/up, Q4_K down, 10 of 64 experts
    "iq3_q4k": Spec(hidden=512, n_experts=64, top_k=10, inter=256, gate_type=O.IQ3_S, up_type=O.IQ3_S,
                    down_type=O.Q4_K, shared_inter=256, seed=5),
    "q6k": Spec(hidden=512, n_experts=16, top_k=2, inter=256, gate_type=O.Q6_K, up_type=O.Q6_K, down_type=O.Q6_K,
                norm=False),
    "q8_0": Spec(hidden=256, n_experts=8, top_k=3, inter=128, gate_type=O.Q8_0, up_type=O.Q8_0, down_type=O.Q8_0),
    # full config-1 width (hidden 2048: eight 256-column pieces), few experts: small batches take
    # the K-split (4 and 8 slices per item) paths of the grouped products
    "iq_wide": Spec(hidden=2048, n_experts=16, top_k=2, inter=512, gate_type=O.IQ2_S, up_type=O.IQ2_S,
                    down_type=O.IQ3_S, shared_inter=512, seed=2),
    # the formats of the reference's own resident file (UD-IQ2_M): IQ2_XXS gate/up, IQ3_XXS down,
    # IQ4_XS shared expert
    "iq_xxs": Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_XXS, up_type=O.IQ2_XXS,
                   down_type=O.IQ3_XXS, shared_inter=256, sh_types=(O.IQ4_XS, O.IQ4_XS, O.IQ4_XS), seed=8),
    "iq4xs": Spec(hidden=768, n_experts=16, top_k=4, inter=512, gate_type=O.IQ3_XXS, up_type=O.IQ3_XXS,
                  down_type=O.IQ4_XS, seed=9),
}


# T = 256 and 1500: piles of 16 and more picks on average take passes of 16 or 32 picks (two or
# four n-tiles per decoded weight fragment); 1500 leaves ragged last passes
@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("T", [1, 5, 64, 256])
@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
def test_moe_forward_matches_oracle(name, T, mode):
    _moe_case(name, T, mode)


@pytest.mark.parametrize("name", ["iq_mix", "iq3_q4k", "mxfp4_gptoss", "iq_xxs"])
@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
def test_moe_forward_prefill_piles(name, mode):
    _moe_case(name, 1500, mode)


def _moe_case(name, T, mode):
    s = SPECS[name]
    L = build_cpu(s)
    x = make_input(s, T)
    ref = O.moe_forward(L, x, mode)
    moe = build_gpu(L, act_mode=mode)
    taps = {}
    out = moe.forward(_t(x)[None], taps=taps)[0].cpu().numpy()
    from coachwhip_b200 import _lib

    _lib.status(0)
    assert np.array_equal(taps["ids"].cpu().numpy().astype(np.uint32), ref["ids"]), "expert ids"
    ulp = np.abs(taps["weights"].cpu().numpy().view(np.int32).astype(np.int64) - ref["w"].view(np.int32))
    assert ulp.max() <= 1, f"routing weights differ by {ulp.max()} ulp"
    op, oh = O.permute(ref["ids"], s.n_experts)
    assert np.array_equal(taps["pairs"].cpu().numpy().view(np.uint32), op)
    assert np.array_equal(taps["heads"].cpu().numpy().reshape(-1).view(np.uint32), oh)
    err = rel_l2(out, ref["out"])
    assert err < RTOL, err


def test_moe_forward_residual_and_dtype():
    s = SPECS["q4k_shared"]
    L = build_cpu(s)
    x = make_input(s, 4)
    ref = O.moe_forward(L, x, O.MODE_CANDLE)
    moe = build_gpu(L)
    r = make_input(s, 4, seed=99)
    out = moe.forward(_t(x)[None], residual=_t(r)[None])[0].cpu().numpy()
    assert rel_l2(out, ref["out"] + r) < RTOL
    xb = _t(x).to(torch.bfloat16)[None]
    ob = moe.forward(xb)
    assert ob.dtype == torch.bfloat16 and ob.shape == (1, 4, s.hidden)


def test_moe_forward_is_deterministic():
    s = SPECS["iq_mix"]
    L = build_cpu(s)
    moe = build_gpu(L)
    x = _t(make_input(s, 64))[None]
    a = moe.forward(x).cpu().numpy()
    b = moe.forward(x).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_moe_forward_skewed_piles():
    # every token picks the same experts: one pile larger than a pass (64 picks)
    s = Spec(hidden=256, n_experts=16, top_k=2, inter=256, gate_type=O.Q4_K, up_type=O.Q4_K, down_type=O.Q4_K)
    L = build_cpu(s)
    L["router_b"] = np.zeros(16, dtype=np.float32)
    L["router_b"][3] = 50.0
    L["router_b"][9] = 49.0
    x = make_input(s, 150)
    ref = O.moe_forward(L, x, O.MODE_CANDLE)
    moe = build_gpu(L)
    out = moe.forward(_t(x)[None])[0].cpu().numpy()
    assert rel_l2(out, ref["out"]) < RTOL
