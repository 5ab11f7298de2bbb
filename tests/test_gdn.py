"""The Gated DeltaNet word step (the linear-attention mixer before the MoE block).

CPU: the oracle's restatement of the reference's fused word kernel (attn_kernel.rs:24-143) against
its restatement of the op-by-op path (model_next.rs:581-620) and against a float64 evaluation of the
delta rule on the input generator of the reference's own test (crates/engine/tests/linear_attention.rs:
9-20, 47-60); the C ABI's argument checks (no device call). GPU: cwx_gdn_word / cwx_delta_word against
the oracle, one word and a run of words carrying the memory, at Qwen3-Next's shape and at ragged ones.

Tolerances (f32 arithmetic in another summation order than the reference kernel's single thread per
column): read-out o and memory within 2e-5 of the largest magnitude, the conv window bit for bit
(it is a copy), 1e-4 over runs of words (the reference test's bar for its two delta-rule forms).
"""

import ctypes

import numpy as np
import pytest

import oracle as O


class Lcg:
    """The reference test's generator (linear_attention.rs:9-20): 64-bit LCG, the top 31 bits of the
    state as a uniform in [-1, 1)."""

    def __init__(self, seed: int):
        self.s = seed

    def next(self) -> np.float32:
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        return np.float32(np.float32(self.s >> 33) / np.float32(1 << 31)) * np.float32(2.0) - np.float32(1.0)

    def tensor(self, shape, scale: float) -> np.ndarray:
        n = int(np.prod(shape))
        return (np.array([self.next() for _ in range(n)], dtype=np.float32) * np.float32(scale)).reshape(shape)


def ref_test_inputs(seed: int, l: int, n_v: int, dk: int, dv: int):
    """linear_attention.rs:47-60: unit q and k, v in [-1, 1), beta = sigmoid(2u), log decay = -0.3|u|."""
    g = Lcg(seed)

    def unit(t):
        return (t / np.sqrt((t * t).sum(axis=2, keepdims=True, dtype=np.float32))).astype(np.float32)

    q = unit(g.tensor((l, n_v, dk), 1.0))
    k = unit(g.tensor((l, n_v, dk), 1.0))
    v = g.tensor((l, n_v, dv), 1.0)
    beta = (1.0 / (1.0 + np.exp(-g.tensor((l, n_v), 2.0)))).astype(np.float32)
    log_decay = (np.abs(g.tensor((l, n_v), 0.3)) * -1.0).astype(np.float32)
    return q, k, v, beta, log_decay


def delta_f64(q, k, v, beta, log_decay, s):
    s = s.astype(np.float64).copy()
    outs = []
    for t in range(q.shape[0]):
        g = np.exp(log_decay[t].astype(np.float64))[:, None, None]
        s = s * g
        sk = np.einsum("hi,hij->hj", k[t].astype(np.float64), s)
        d = (v[t] - sk) * beta[t][:, None]
        s = s + np.einsum("hi,hj->hij", k[t].astype(np.float64), d)
        outs.append(np.einsum("hi,hij->hj", q[t].astype(np.float64), s))
    return np.stack(outs), s


def layer_inputs(seed: int, n_k, n_v, dk, dv, taps, n_seq=1):
    """Seeded synthetic layer constants and per-word tensors of the shapes the reference reads."""
    rng = np.random.default_rng(seed)
    ch = 2 * n_k * dk + n_v * dv
    f = np.float32
    consts = dict(conv_w=(rng.standard_normal((ch, taps)) * 0.4).astype(f),
                  dt_bias=rng.standard_normal(n_v).astype(f),
                  a=(-np.exp(rng.uniform(0.0, np.log(16.0), n_v))).astype(f),
                  norm_w=(1.0 + 0.1 * rng.standard_normal(dv)).astype(f))
    words = dict(qkv=rng.standard_normal((n_seq, ch)).astype(f), z=rng.standard_normal((n_seq, n_v * dv)).astype(f),
                 ba=rng.standard_normal((n_seq, 2 * n_v)).astype(f),
                 conv_state=rng.standard_normal((n_seq, taps - 1, ch)).astype(f),
                 s=(0.1 * rng.standard_normal((n_seq, n_v, dk, dv))).astype(f))
    return consts, words


def close(a, b, tol):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() <= tol * max(1.0, np.abs(b).max())


@pytest.mark.parametrize("shape", [(2, 4, 16, 24, 4, 0), (2, 4, 16, 24, 4, 1), (1, 3, 8, 6, 2, 0), (4, 8, 32, 40, 3, 1)])
def test_fused_restatement_matches_op_by_op(shape):
    n_k, n_v, dk, dv, taps, cyc = shape
    c, w = layer_inputs(1, n_k, n_v, dk, dv, taps)
    args = (w["qkv"][0], w["z"][0], w["ba"][0], w["conv_state"][0], c["conv_w"], c["dt_bias"], c["a"], c["norm_w"],
            w["s"][0])
    fo, fs, fc = O.gdn_word(n_k, n_v, dk, dv, taps, cyc, 1e-6, *args)
    po, ps, pc = O.gdn_word(n_k, n_v, dk, dv, taps, cyc, 1e-6, *args, ops=True)
    assert close(fo, po, 2e-5) and close(fs, ps, 2e-5)
    assert np.array_equal(fc, pc)
    # the window moved one word on: rows 1.. then the new word
    assert np.array_equal(fc[:-1], w["conv_state"][0][1:]) and np.array_equal(fc[-1], w["qkv"][0])


@pytest.mark.parametrize("l,seed", [(1, 1), (7, 2), (64, 3)])
def test_delta_steps_on_the_reference_tests_inputs(l, seed):
    n_v, dk, dv = 3, 8, 6  # linear_attention.rs:64
    q, k, v, beta, log_decay = ref_test_inputs(seed, l, n_v, dk, dv)
    s0 = np.zeros((n_v, dk, dv), np.float32)
    o, s = O.delta_steps(q, k, v, beta, log_decay, s0)
    o64, s64 = delta_f64(q, k, v, beta, log_decay, s0)
    assert np.abs(o - o64).max() < 1e-5 and np.abs(s - s64).max() < 1e-5


def test_gdn_abi_checks_arguments_before_any_device_call():
    from coachwhip_b200 import _lib

    L = _lib.lib()
    fake = 4096  # non-null addresses that are never dereferenced: every case fails before a launch
    ok = _lib.GdnLayer(2, 4, 16, 16, 4, 0, 1e-6, fake, fake, fake, fake)

    def call(layer, n_seq=1, conv_state=fake, conv_out=fake + 64):
        return L.cwx_gdn_word(ctypes.byref(layer), n_seq, fake, fake, fake, conv_state, fake, fake, fake, conv_out, None)

    assert call(_lib.GdnLayer(3, 4, 16, 16, 4, 0, 1e-6, fake, fake, fake, fake)) == _lib.EINVAL  # n_v % n_k
    assert call(_lib.GdnLayer(2, 4, 16, 16, 1, 0, 1e-6, fake, fake, fake, fake)) == _lib.EINVAL  # taps < 2
    assert call(_lib.GdnLayer(2, 4, 16, 288, 4, 0, 1e-6, fake, fake, fake, fake)) == _lib.EUNSUPPORTED
    assert call(_lib.GdnLayer(2, 4, 640, 16, 4, 0, 1e-6, fake, fake, fake, fake)) == _lib.EUNSUPPORTED
    assert call(ok, n_seq=-1) == _lib.EINVAL
    assert call(ok, conv_out=fake) == _lib.EINVAL
    assert b"conv_out must be a buffer of its own" in L.cwx_last_error()
    assert call(ok, n_seq=0) == _lib.OK  # nothing to do
    assert L.cwx_delta_word(4, 600, 8, fake, fake, fake, fake + 64, None) == _lib.EUNSUPPORTED
    assert L.cwx_delta_word(4, 8, 8, fake, fake, fake, fake, None) == _lib.EINVAL


def test_python_mirror_keeps_the_reference_errors():
    import torch

    from coachwhip_b200.gdn import GdnWord, gdn_word

    t = torch.zeros(4, dtype=torch.float64)
    op = GdnWord(t, t, t, t, t, t, 1, 1, 2, 2, 2, False, 1e-6)
    with pytest.raises(RuntimeError, match="coachwhip-gdn-word: conv_state must be f32"):
        gdn_word(op, t, t, t, t)


# ---------------------------------------------------------------- GPU


def _gpu_word(c, w, n_k, n_v, dk, dv, taps, cyc, eps=1e-6, in_place=False):
    import torch

    from coachwhip_b200.gdn import GdnWord, gdn_word

    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    n_seq = w["qkv"].shape[0]
    op = GdnWord(d(w["conv_state"]), d(c["conv_w"]), d(c["dt_bias"]), d(c["a"]), d(c["norm_w"]), d(w["s"]), n_k, n_v,
                 dk, dv, taps, bool(cyc), eps)
    o, s, cv = gdn_word(op, d(w["qkv"]), d(w["z"]), d(w["ba"][:, :n_v]), d(w["ba"][:, n_v:]),
                        s_out=op.s if in_place else None)
    torch.cuda.synchronize()
    return o.cpu().numpy().reshape(n_seq, -1), s.cpu().numpy(), cv.cpu().numpy()


def _oracle_word(c, w, i, n_k, n_v, dk, dv, taps, cyc, eps=1e-6):
    return O.gdn_word(n_k, n_v, dk, dv, taps, cyc, eps, w["qkv"][i], w["z"][i], w["ba"][i], w["conv_state"][i],
                      c["conv_w"], c["dt_bias"], c["a"], c["norm_w"], w["s"][i])


GDN_SHAPES = [
    # n_k, n_v, dk, dv, taps, cycle, n_seq
    (16, 32, 128, 128, 4, 1, 1),  # Qwen3-Next / Qwen3.6 shape, key heads cycled
    (16, 32, 128, 128, 4, 0, 3),  # key heads side by side, three sequences
    (2, 6, 40, 72, 3, 1, 2),      # ragged: a last CTA of 8 columns, rows not a multiple of 8
    (1, 2, 256, 256, 4, 0, 1),    # 32 rows per warp, clusters of 8 CTAs
    (1, 1, 512, 32, 2, 0, 1),     # 64 rows per warp, two taps
    (1, 1, 8, 1, 2, 0, 2),        # one column
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", GDN_SHAPES)
def test_gdn_word_matches_oracle(shape):
    n_k, n_v, dk, dv, taps, cyc, n_seq = shape
    c, w = layer_inputs(11, n_k, n_v, dk, dv, taps, n_seq)
    go, gs, gc = _gpu_word(c, w, n_k, n_v, dk, dv, taps, cyc)
    for i in range(n_seq):
        oo, os_, oc = _oracle_word(c, w, i, n_k, n_v, dk, dv, taps, cyc)
        assert close(go[i], oo, 2e-5), np.abs(go[i] - oo).max()
        assert close(gs[i], os_, 2e-5), np.abs(gs[i] - os_).max()
        assert np.array_equal(gc[i], oc)


@pytest.mark.gpu
def test_gdn_words_carry_the_memory_in_place():
    import torch

    from coachwhip_b200.gdn import GdnWord, gdn_word

    n_k, n_v, dk, dv, taps, cyc, n_seq, L = 16, 32, 128, 128, 4, 1, 2, 16
    c, w = layer_inputs(5, n_k, n_v, dk, dv, taps, n_seq)
    rng = np.random.default_rng(6)
    ch = 2 * n_k * dk + n_v * dv
    words = [dict(qkv=rng.standard_normal((n_seq, ch)).astype(np.float32),
                  z=rng.standard_normal((n_seq, n_v * dv)).astype(np.float32),
                  ba=rng.standard_normal((n_seq, 2 * n_v)).astype(np.float32)) for _ in range(L)]
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    op = GdnWord(d(w["conv_state"]), d(c["conv_w"]), d(c["dt_bias"]), d(c["a"]), d(c["norm_w"]), d(w["s"]), n_k, n_v,
                 dk, dv, taps, True, 1e-6)
    ref_s = [w["s"][i].copy() for i in range(n_seq)]
    ref_c = [w["conv_state"][i].copy() for i in range(n_seq)]
    for x in words:
        o, s, cv = gdn_word(op, d(x["qkv"]), d(x["z"]), d(x["ba"][:, :n_v]), d(x["ba"][:, n_v:]), s_out=op.s)
        assert s.data_ptr() == op.s.data_ptr()
        op.conv_state = cv
        go = o.cpu().numpy()
        for i in range(n_seq):
            oo, ref_s[i], ref_c[i] = O.gdn_word(n_k, n_v, dk, dv, taps, cyc, 1e-6, x["qkv"][i], x["z"][i], x["ba"][i],
                                                ref_c[i], c["conv_w"], c["dt_bias"], c["a"], c["norm_w"], ref_s[i])
            assert close(go[i], oo, 1e-4)
    gs = op.s.cpu().numpy()
    for i in range(n_seq):
        assert close(gs[i], ref_s[i], 1e-4)
        assert np.array_equal(op.conv_state.cpu().numpy()[i], ref_c[i])


@pytest.mark.gpu
@pytest.mark.parametrize("l,seed,shape", [(8, 1, (3, 8, 6)), (4, 2, (32, 128, 128)), (2, 3, (5, 200, 40))])
def test_delta_word_matches_word_by_word(l, seed, shape):
    import torch

    from coachwhip_b200.gdn import delta_word

    n_v, dk, dv = shape
    q, k, v, beta, log_decay = ref_test_inputs(seed, l, n_v, dk, dv) if dk * n_v <= 2048 else (
        *(x.astype(np.float32) for x in _unit_inputs(seed, l, n_v, dk, dv)),)
    s = torch.zeros(n_v, dk, dv, device="cuda")
    ref_s = np.zeros((n_v, dk, dv), np.float32)
    for t in range(l):
        decay = np.exp(log_decay[t]).astype(np.float32)
        d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
        o, s = delta_word(d(q[t]), d(k[t]), d(v[t]), d(beta[t]), d(decay), s)
        oo, ref_s = O.delta_steps(q[t:t + 1], k[t:t + 1], v[t:t + 1], beta[t:t + 1], log_decay[t:t + 1], ref_s)
        assert close(o.cpu().numpy(), oo[0], 1e-4)
    assert close(s.cpu().numpy(), ref_s, 1e-4)


def _unit_inputs(seed, l, n_v, dk, dv):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((l, n_v, dk))
    k = rng.standard_normal((l, n_v, dk))
    q /= np.linalg.norm(q, axis=2, keepdims=True)
    k /= np.linalg.norm(k, axis=2, keepdims=True)
    return (q, k, rng.uniform(-1, 1, (l, n_v, dv)), 1 / (1 + np.exp(-2 * rng.uniform(-1, 1, (l, n_v)))),
            -0.3 * np.abs(rng.uniform(-1, 1, (l, n_v))))
