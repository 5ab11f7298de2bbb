"""The gated full-attention word step (FullAttn::forward between the projections).

CPU: the oracle's restatement (model_next.rs:666-720) against a float64 evaluation of the same
formulas, and the C ABI's argument checks (no device call). GPU: cwx_attn_word against the oracle
at Qwen3-Next's shape (16 query heads over 2 kv heads of 256, rope on 64) and others, cache
lengths on both sides of the 32-row chunks, several sequences of different lengths, a grid large
enough that each CTA walks several chunks, a run of words appended one after another.

Tolerance: the split-K softmax merges 32-row chunks (exp(s - m_chunk) rescaled by exp(m_chunk - M))
where the reference normalises once, and sums in another order: outputs within 2e-5 of the largest
magnitude; the appended cache rows (normalised and rotated k, copied v) within 1e-6.
"""

import ctypes

import numpy as np
import pytest

import oracle as O


def attn_f64(n_head, n_kv, hd, rot, eps, base, L, pos, qg, k_new, v_new, qw, kw, kc, vc):
    g = n_head // n_kv

    def norm_rope(x, w):
        x = x.astype(np.float64)
        y = x / np.sqrt((x * x).mean() + eps) * w
        half = rot // 2
        inv = 1.0 / base ** (2.0 * np.arange(half) / rot)
        f = pos * inv
        a, b = y[:half].copy(), y[half:rot].copy()
        y[:half] = a * np.cos(f) - b * np.sin(f)
        y[half:rot] = a * np.sin(f) + b * np.cos(f)
        return y

    kc = kc.astype(np.float64).copy()
    vc = vc.astype(np.float64).copy()
    for kv in range(n_kv):
        kc[kv, L] = norm_rope(k_new[kv], kw)
        vc[kv, L] = v_new[kv]
    out = np.empty((n_head, hd))
    for h in range(n_head):
        q = norm_rope(qg[h, :hd], qw)
        s = kc[h // g, :L + 1] @ q / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = (p @ vc[h // g, :L + 1]) / (1 + np.exp(-qg[h, hd:].astype(np.float64)))
    return out.reshape(-1), kc, vc


def inputs(seed, n_head, n_kv, hd, cap, n_seq=1):
    rng = np.random.default_rng(seed)
    f = np.float32
    return dict(qg=rng.standard_normal((n_seq, n_head, 2 * hd)).astype(f),
                k_new=rng.standard_normal((n_seq, n_kv, hd)).astype(f),
                v_new=rng.standard_normal((n_seq, n_kv, hd)).astype(f),
                qw=(1 + 0.1 * rng.standard_normal(hd)).astype(f), kw=(1 + 0.1 * rng.standard_normal(hd)).astype(f),
                kc=(0.5 * rng.standard_normal((n_seq, n_kv, cap, hd))).astype(f),
                vc=rng.standard_normal((n_seq, n_kv, cap, hd)).astype(f))


def close(a, b, tol):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.abs(a - b).max() <= tol * max(1.0, np.abs(b).max())


@pytest.mark.parametrize("shape,L", [((4, 2, 64, 16), 0), ((4, 2, 64, 16), 9), ((16, 2, 256, 64), 70),
                                     ((6, 3, 128, 128), 33)])
def test_oracle_matches_float64(shape, L):
    n_head, n_kv, hd, rot = shape
    w = inputs(1, n_head, n_kv, hd, 80)
    args = (n_head, n_kv, hd, rot, 1e-6, 1e7, L, L + 3, w["qg"][0], w["k_new"][0], w["v_new"][0], w["qw"], w["kw"])
    o, kc, vc = O.attn_word(*args, w["kc"][0], w["vc"][0])
    o64, kc64, vc64 = attn_f64(*args, w["kc"][0], w["vc"][0])
    assert close(o, o64, 1e-5)
    assert close(kc, kc64, 1e-6) and np.array_equal(vc, vc64.astype(np.float32))
    # rows other than L are untouched
    assert np.array_equal(np.delete(kc, L, axis=1), np.delete(w["kc"][0], L, axis=1))


def test_attn_abi_checks_arguments_before_any_device_call():
    from coachwhip_b200 import _lib

    lib = _lib.lib()
    fake = 4096  # non-null addresses that are never dereferenced: every case fails before a launch

    def call(n_head=16, n_kv=2, hd=256, rot=64, n_seq=1, cap=64, ctx=None):
        L = _lib.AttnLayer(n_head, n_kv, hd, rot, 1e-6, 1e7, fake, fake)
        return lib.cwx_attn_word(ctx, ctypes.byref(L), n_seq, cap, fake, fake, fake, fake, fake, fake, fake, fake,
                                 None)

    assert call(n_head=15) == _lib.EINVAL
    assert call(n_head=34, n_kv=2) == _lib.EUNSUPPORTED  # 17 query heads per kv head
    assert call(hd=96) == _lib.EUNSUPPORTED
    assert call(rot=65) == _lib.EINVAL and call(rot=258) == _lib.EINVAL
    assert call(cap=0) == _lib.EINVAL
    assert call() == _lib.EINVAL  # null context
    assert b"null context" in lib.cwx_last_error()


# ---------------------------------------------------------------- GPU

SHAPES = [
    # n_head, n_kv, hd, rot, cap, lengths of the sequences
    (16, 2, 256, 64, 200, [0]),
    (16, 2, 256, 64, 200, [31, 32, 33]),
    (16, 2, 256, 64, 1100, [1000]),
    (8, 2, 128, 128, 300, [5, 130, 299]),
    (16, 1, 64, 32, 128, [127, 1]),
    (2, 2, 64, 0, 64, [40]),
    # a grid of 8 x 2 x 256 chunks: several 32-row chunks per CTA (online softmax across them)
    (16, 2, 256, 64, 8192, [8191, 96, 95, 0, 4000, 97, 191, 192]),
]


def _gpu(att_shape, w, lens, pos):
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200.attn import FullAttn, KvCache, attn_word

    n_head, n_kv, hd, rot, cap = att_shape
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    att = FullAttn(d(w["qw"]), d(w["kw"]), n_head, n_kv, hd, rot, 1e7, 1e-6)
    cache = KvCache(len(lens), n_kv, cap, hd, "cuda")
    cache.k.copy_(d(w["kc"]))
    cache.v.copy_(d(w["vc"]))
    cache.len.copy_(torch.tensor(lens, dtype=torch.int32))
    out = attn_word(att, cache, d(w["qg"]), d(w["k_new"]), d(w["v_new"]),
                    pos=torch.tensor(pos, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    _lib.status(0)
    return out.cpu().numpy(), cache


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES)
def test_attn_word_matches_oracle(shape):
    n_head, n_kv, hd, rot, cap, lens = shape
    w = inputs(7, n_head, n_kv, hd, cap, len(lens))
    pos = [l_ + 11 for l_ in lens]
    go, cache = _gpu((n_head, n_kv, hd, rot, cap), w, lens, pos)
    kc, vc = cache.k.cpu().numpy(), cache.v.cpu().numpy()
    for i, L in enumerate(lens):
        oo, okc, ovc = O.attn_word(n_head, n_kv, hd, rot, 1e-6, 1e7, L, pos[i], w["qg"][i], w["k_new"][i],
                                   w["v_new"][i], w["qw"], w["kw"], w["kc"][i], w["vc"][i])
        assert close(go[i], oo, 2e-5), np.abs(go[i] - oo).max()
        assert close(kc[i], okc, 1e-6) and np.array_equal(vc[i], ovc)
    assert cache.len.cpu().tolist() == [l_ + 1 for l_ in lens]


@pytest.mark.gpu
def test_attn_words_append_to_the_cache():
    import torch

    from coachwhip_b200.attn import FullAttn, KvCache, attn_word

    n_head, n_kv, hd, rot, cap, n_seq, words = 16, 2, 256, 64, 96, 2, 70
    rng = np.random.default_rng(3)
    qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    att = FullAttn(d(qw), d(kw), n_head, n_kv, hd, rot, 1e7, 1e-6)
    cache = KvCache(n_seq, n_kv, cap, hd, "cuda")
    ref_k = np.zeros((n_seq, n_kv, cap, hd), np.float32)
    ref_v = np.zeros_like(ref_k)
    for t in range(words):
        qg = rng.standard_normal((n_seq, n_head, 2 * hd)).astype(np.float32)
        kn = rng.standard_normal((n_seq, n_kv, hd)).astype(np.float32)
        vn = rng.standard_normal((n_seq, n_kv, hd)).astype(np.float32)
        go = attn_word(att, cache, d(qg), d(kn), d(vn)).cpu().numpy()
        for i in range(n_seq):
            oo, ref_k[i], ref_v[i] = O.attn_word(n_head, n_kv, hd, rot, 1e-6, 1e7, t, t, qg[i], kn[i], vn[i], qw, kw,
                                                 ref_k[i], ref_v[i])
            assert close(go[i], oo, 2e-5), (t, np.abs(go[i] - oo).max())
    assert close(cache.k.cpu().numpy(), ref_k, 1e-6)


@pytest.mark.gpu
def test_attn_word_reports_a_full_cache():
    from coachwhip_b200 import CwxError

    w = inputs(1, 4, 2, 64, 8)
    with pytest.raises(CwxError, match="attention cache row"):
        _gpu((4, 2, 64, 16, 8), w, [8], [8])  # len == cap: no row left
