"""Routing margins on the benchmark configurations' seeded inputs (CPU only).

The reference computes router logits as an f32 GEMV in the gemm crate (candle's CPU matmul),
whose summation order is not restated here; the library and the oracle both take the exact
products of the f32 inputs summed in f64 and rounded once. The expert ids are the same under both
definitions wherever, for each token, the gap between its k-th and (k+1)-th logit exceeds the
f32 GEMV's rounding error on those two logits.

What this test establishes on layer 0 of each configuration, every token:
  1. The ids of six f32 summation orders (sequential, sequential FMA, 8 and 16 strided lanes,
     256-column blocks, pairwise) equal the oracle's ids: the routing does not depend on the
     order on these inputs.
  2. The margin statistics. The rigorous worst-case bound of an f32 dot over H terms,
     gamma_H * sum|x_i w_i| with gamma_H = H u / (1 - H u), u = 2^-24, is about 3.5e-3 here,
     while the k-th to (k+1)-th gaps of Gaussian logits have a median near 0.04 and an
     exponential-like lower tail: no token reaches a gap of 100x that bound (0 %), and about 85 %
     reach 1x. Against the largest error actually seen over the six orders (about 1e-5), the
     gap exceeds 100x for 93-100 % of the tokens of each configuration; those fractions are
     asserted as measured, and the few tokens below it are the ones item 1 checks directly.
"""

import numpy as np
import pytest

import oracle as O

U = 2.0 ** -24
T_RW, T_RB, T_IN = 3, 4, 12


def _normal(seed, layer, t, n, std):
    return O.normal(O.stream(seed, layer, t), 0, n, std)


def _zipf(E, s, seed):
    r = np.random.default_rng(seed).permutation(E) + 1
    return (-s * np.log(r) - np.log(np.sum(np.arange(1, E + 1, dtype=np.float64) ** -s))).astype(np.float32)


# name: (H, E, k, weight seed, input seed, T, router bias, zipf, min fraction with gap > 100x seen error)
CASES = {
    "C0": (2048, 256, 8, 0, 1, 64, False, 0.0, 1.0),
    "C1": (2048, 256, 8, 2, 2, 64, False, 0.0, 0.90),
    "C2": (2048, 256, 8, 2, 3, 4096, False, 0.0, 0.95),
    "C3": (2880, 128, 4, 4, 5, 4096, True, 0.0, 0.95),
    "C4": (2048, 512, 10, 5, 6, 8192, False, 1.1, 0.95),
}


@pytest.mark.parametrize("name", list(CASES))
def test_routing_margin_and_order_independence(name):
    H, E, k, ws, xs, T, rbias, zipf, min_frac = CASES[name]
    W = _normal(ws, 0, T_RW, E * H, 0.02).reshape(E, H)
    x = _normal(xs, 0, T_IN, T * H, 1.0).reshape(T, H)
    b = _normal(ws, 0, T_RB, E, 0.02) if rbias else None
    if zipf:
        b = _zipf(E, zipf, ws)
    lg = O.router(x, W, b)
    ids, _ = O.route(lg, k, True)

    # 1. every f32 summation order routes every token to the same experts
    errs = []
    exact = x.astype(np.float64) @ W.astype(np.float64).T
    for order in range(O.ROUTER_ORDERS):
        lf = O.router_f32(x, W, b, order)
        fi, _ = O.route(lf, k, True)
        bad = np.nonzero((np.sort(fi, 1) != np.sort(ids, 1)).any(1))[0]
        assert bad.size == 0, f"{name}: order {order} routes tokens {bad[:8].tolist()} differently"
        eb = 0.0 if b is None else b.astype(np.float64)
        errs.append(np.abs(lf.astype(np.float64) - (exact + eb)).max())
    seen = max(errs)

    # 2. margins against the rigorous bound and against the error seen
    full = exact + (0.0 if b is None else b.astype(np.float64))
    order_ = np.argsort(-full, axis=1, kind="stable")
    r = np.arange(T)
    a, c = order_[:, k - 1], order_[:, k]
    gap = full[r, a] - full[r, c]
    gamma = H * U / (1 - H * U)
    absum = np.abs(x.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    bound = gamma * np.maximum(absum[r, a], absum[r, c])
    frac_rigorous = float(np.mean(gap > 2 * bound))
    frac_100x_rigorous = float(np.mean(gap > 200 * bound))
    frac_100x_seen = float(np.mean(gap > 200 * seen))
    print(f"{name}: T={T} median gap {np.median(gap):.3e}, rigorous bound <= {bound.max():.3e}, "
          f"seen error {seen:.3e}; gap > 2x bound: {frac_rigorous:.3f}, > 200x bound: {frac_100x_rigorous:.3f}, "
          f"> 200x seen: {frac_100x_seen:.3f}")
    assert frac_100x_seen >= min_frac, (name, frac_100x_seen)
    assert frac_rigorous > 0.75
