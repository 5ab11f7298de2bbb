"""CPU checks of the oracle: its dequantisation against ggml's gguf package, its route() against
the reference's known answers, and the invariants of its piles, quantisers and generator."""

import numpy as np
import pytest

import oracle as O

FORMATS = [O.Q4_K, O.Q6_K, O.Q8_0, O.MXFP4, O.IQ2_S, O.IQ3_S, O.IQ2_XXS, O.IQ3_XXS, O.IQ4_XS]


def _gguf_type(fmt):
    from gguf.constants import GGMLQuantizationType as G

    return {O.Q4_K: G.Q4_K, O.Q6_K: G.Q6_K, O.Q8_0: G.Q8_0, O.MXFP4: G.MXFP4, O.IQ2_S: G.IQ2_S,
            O.IQ3_S: G.IQ3_S, O.IQ2_XXS: G.IQ2_XXS, O.IQ3_XXS: G.IQ3_XXS, O.IQ4_XS: G.IQ4_XS}[fmt]


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequant_matches_gguf_package(fmt):
    gq = pytest.importorskip("gguf.quants")
    x = O.normal(O.stream(9, fmt, 1), 0, 256 * 40, 0.02)
    x[:256] *= 100.0
    x[256:512] = 0.0
    q = O.quantize(fmt, x)
    got = O.dequantize(fmt, q, x.size)
    want = gq.dequantize(q, _gguf_type(fmt)).reshape(-1).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q8_0_quantiser_matches_gguf_package():
    gq = pytest.importorskip("gguf.quants")
    x = O.normal(O.stream(9, 8, 2), 0, 32 * 64, 1.0)
    got = O.quantize(O.Q8_0, x)
    want = gq.quantize(x.reshape(-1, 32), _gguf_type(O.Q8_0)).reshape(-1)
    # gguf rounds x*id with numpy's round-half-to-even; candle rounds half away from zero.
    assert (got != want).mean() < 1e-3


@pytest.mark.parametrize("fmt", FORMATS)
def test_quantisers_round_trip(fmt):
    x = O.normal(O.stream(1, fmt, 5), 0, 256 * 64, 0.02)
    y = O.dequantize(fmt, O.quantize(fmt, x), x.size)
    err = np.linalg.norm(y - x) / np.linalg.norm(x)
    bound = {O.Q4_K: 0.12, O.Q6_K: 0.03, O.Q8_0: 0.01, O.MXFP4: 0.15, O.IQ2_S: 0.45, O.IQ3_S: 0.4, O.IQ2_XXS: 0.5,
             O.IQ3_XXS: 0.3, O.IQ4_XS: 0.12}[fmt]
    assert err < bound, err


def test_q8k_quantiser_semantics():
    # k_quants.rs:2495-2534: max by |x| (first on ties), iscale = -127/max, bsums over 16
    x = np.zeros(256, dtype=np.float32)
    x[3], x[7] = -2.0, 2.0
    x[10] = 1.0
    q = O.quantize(O.Q8_K, x)
    d = q[:4].view(np.float32)[0]
    qs = q[4:260].view(np.int8)
    assert d == np.float32(1.0) / (np.float32(-127.0) / np.float32(-2.0))
    assert qs[3] == -127 and qs[7] == 127 and qs[10] == 64  # max is x[3] (first on ties); round(63.5) = 64
    bsums = q[260:292].view(np.int16)
    assert bsums[0] == qs[:16].sum()


ROUTE_KATS = [  # crates/engine/tests/router.rs:21-60, lookahead.rs:6-20
    ([[0.1, 3.0, 2.0, -1.0, 1.0]], 3, True, [[1, 2, 4]]),
    ([[5.0, 0.0, 1.0, 2.0], [0.0, 1.0, 9.0, 3.0]], 2, True, [[0, 3], [2, 3]]),
    ([[0.1, 3.0, 2.0, -1.0, 1.0]], 5, False, [[1, 2, 4, 0, 3]]),
    ([[1.0, 1.0, 2.0, 1.0]], 4, False, [[2, 0, 1, 3]]),
    ([[0.5] * 6], 6, False, [[0, 1, 2, 3, 4, 5]]),
]


def _softmax(row):
    m = np.float32(max(row))
    e = np.exp(np.asarray(row, dtype=np.float32) - m)
    return e / e.sum()


@pytest.mark.parametrize("case", range(len(ROUTE_KATS)))
def test_route_known_answers(case):
    logits, k, norm, want = ROUTE_KATS[case]
    ids, _ = O.route(np.asarray(logits, dtype=np.float32), k, norm)
    assert ids.tolist() == want


def test_route_renormalised_weights():
    # router.rs:33-44: weights sum to 1 and keep the ratios of the probabilities
    row = [0.5, 2.0, 1.0, -0.5, 1.5]
    ids, w = O.route(np.asarray([row], dtype=np.float32), 3, True)
    p = _softmax(row)
    kept = p[1] + p[4] + p[2]
    assert abs(w.sum() - 1) < 1e-5
    for got, i in zip(w[0], [1, 4, 2]):
        assert abs(got - p[i] / kept) < 1e-5


def test_route_without_renorm_gives_probabilities():
    # router.rs:46-53
    row = [1.0, 0.0, 3.0, 2.0]
    _, w = O.route(np.asarray([row], dtype=np.float32), 2, False)
    p = _softmax(row)
    assert abs(w[0, 0] - p[2]) < 1e-5 and abs(w[0, 1] - p[3]) < 1e-5 and w.sum() < 1.0


def test_route_weights_follow_pick_order():
    # router.rs:55-60
    _, w = O.route(np.asarray([[0.0, 4.0, 1.0, 2.0, 3.0]], dtype=np.float32), 4, True)
    assert np.all(np.diff(w[0]) <= 0)


def test_route_rank_covers_every_expert():
    # lookahead.rs:22-29
    scores = np.array([((i * 7919) % 97) * 0.01 for i in range(512)], dtype=np.float32)[None, :]
    ids, _ = O.route(scores, 512, False)
    assert np.all(np.diff(scores[0][ids[0]]) <= 0)
    assert sorted(ids[0].tolist()) == list(range(512))


def test_piles_are_stable_and_complete():
    rng = np.random.default_rng(0)
    E, T, k = 40, 33, 5
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    pairs, heads = O.permute(ids, E)
    h = heads.reshape(E, 3)
    assert h[:, 2].sum() == T * k
    assert sorted(pairs.tolist()) == list(range(T * k))
    flat = ids.reshape(-1)
    for e in range(E):
        run = pairs[h[e, 1]:h[e, 1] + h[e, 2]]
        assert np.all(flat[run] == e) and np.all(np.diff(run) > 0)


def test_avx_sum_order_is_not_sequential():
    # the softmax denominator follows candle's AVX lane order, not a left-to-right sum
    x = np.array([1e8] + [1.0] * 63, dtype=np.float32)
    _, w = O.route(np.log(x)[None, :], 1, False)
    assert w.shape == (1, 1)


def test_generator_statistics_and_determinism():
    z = O.normal(O.stream(2, 0, 0), 0, 1 << 18)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    a = O.normal(O.stream(2, 0, 0), 1000, 10)
    assert np.array_equal(a, z[1000:1010])


def test_synth_matrix_slices_agree():
    key = O.stream(2, 1, 0)
    whole = O.synth_matrix(O.IQ2_S, key, 0, 3, 64, 512, 0.02)
    part = O.synth_matrix(O.IQ2_S, key, 1, 2, 64, 512, 0.02)
    assert np.array_equal(whole[whole.size // 3:], part)


def test_matmul_modes_bracket_the_quantisation_gap():
    from tests.layers import rel_l2

    key = O.stream(0, 0, 0)
    q = O.synth_matrix(O.Q4_K, key, 0, 1, 64, 2048, 0.02)
    x = O.normal(O.stream(1, 0, 12), 0, 4 * 2048).reshape(4, 2048)
    bpe = 64 * O.row_bytes(O.Q4_K, 2048)
    o1 = O.matmul(O.Q4_K, O.MODE_CANDLE, q, 64, 2048, bpe, 0, x)
    o2 = O.matmul(O.Q4_K, O.MODE_F32, q, 64, 2048, bpe, 0, x)
    gap = rel_l2(o1, o2)
    assert 1e-3 < gap < 2e-2  # the Q8_K activation error, visible and bounded


def test_moe_forward_small_layer_modes():
    from tests.layers import Spec, build_cpu, make_input, rel_l2

    s = Spec(hidden=256, n_experts=8, top_k=2, inter=256, gate_type=O.IQ2_S, up_type=O.IQ2_S,
             down_type=O.IQ3_S, shared_inter=256)
    L = build_cpu(s)
    x = make_input(s, 6)
    a = O.moe_forward(L, x, O.MODE_CANDLE)
    b = O.moe_forward(L, x, O.MODE_F32)
    assert np.array_equal(a["ids"], b["ids"])
    assert rel_l2(a["routed"], b["routed"]) < 1e-5  # IQ matrices use f32 activations in both
    assert rel_l2(a["shared"], b["shared"]) > 1e-4  # the Q4_K shared expert does not
    assert np.allclose(a["out"], a["routed"] + a["shared"])


@pytest.mark.parametrize("types", [(O.IQ2_S, O.IQ2_S, O.IQ3_S), (O.Q4_K, O.Q4_K, O.Q4_K), (O.IQ3_S, O.IQ3_S, O.Q4_K)])
def test_fast_cpu_layer_agrees_with_oracle(types):
    # the vectorised CPU baseline computes the same layer as O1 (candle policy): same routing on
    # these inputs, outputs within the layer bar (the reordered f32 sums can flip a Q8_K code of
    # a down matrix's activations, ~1e-4)
    from tests.layers import Spec, build_cpu, make_input, rel_l2

    s = Spec(hidden=512, n_experts=16, top_k=4, inter=256, gate_type=types[0], up_type=types[1],
             down_type=types[2], shared_inter=256, seed=3)
    L = build_cpu(s)
    x = make_input(s, 24)
    ref = O.moe_forward(L, x, O.MODE_CANDLE)
    got = O.moe_forward_fast(L, x)
    assert rel_l2(got, ref["out"]) < 1e-3
