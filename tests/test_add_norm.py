"""Residual add + RMSNorm after the combine (add_norm, crates/engine/src/fuse_kernel.rs:433-471;
its caller's residual step crates/engine/src/model_next.rs:1432-1436).

Bars: the sum a + b (+ c) bit-exact (three f32 adds in the reference's order); the normalised
output within 1e-5 relative per element of the oracle (candle's CPU RmsNorm, whose f32
left-to-right sum of squares the kernel replaces with an f64 sum rounded once) and within 8 ulp
of the exact (f64) value; the fused form inside cwx_moe_forward bit-exact to the standalone call
on the layer's own output, and within relative L2 1e-3 of the oracle's whole layer.
"""

import ctypes

import numpy as np
import pytest

import oracle as O
from tests.layers import Spec, build_cpu, build_gpu, make_input, rel_l2

EPS = 1e-6
NORM_RTOL = 1e-5  # per element vs the oracle's f32 sum of squares


def _py_add_norm(a, b, c, alpha, eps):
    """candle's RmsNorm restated in plain Python float32 steps (small cases only)."""
    f = np.float32
    s = (a + b) if c is None else ((a + b) + c)
    out = np.empty_like(s)
    for r in range(s.shape[0]):
        sum2 = f(0.0)
        for v in s[r]:
            sum2 = f(sum2 + f(v * v))
        m = f(np.sqrt(f(f(sum2 / f(s.shape[1])) + f(eps))))
        out[r] = (s[r] / m) * alpha
    return s, out


def _exact(s, alpha, eps):
    s64 = s.astype(np.float64)
    m = np.sqrt((s64 * s64).sum(axis=1, keepdims=True) / s.shape[1] + eps)
    return s64 / m * alpha.astype(np.float64)


def _inputs(rows, H, seed, with_c=True):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((rows, H), dtype=np.float32)
    b = (rng.standard_normal((rows, H), dtype=np.float32) * 0.5).astype(np.float32)
    c = rng.standard_normal((rows, H), dtype=np.float32) if with_c else None
    alpha = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    return a, b, c, alpha


@pytest.mark.parametrize("rows,H,with_c", [(3, 37, True), (2, 64, False), (4, 256, True)])
def test_oracle_matches_plain_restatement(rows, H, with_c):
    a, b, c, alpha = _inputs(rows, H, 11 + H, with_c)
    s, o = O.add_rms_norm(a, b, c, alpha, EPS)
    ps, po = _py_add_norm(a, b, c, alpha, EPS)
    assert np.array_equal(s.view(np.uint32), ps.view(np.uint32))
    assert np.array_equal(o.view(np.uint32), po.view(np.uint32))


def test_abi_rejects_bad_arguments_without_a_device():
    from coachwhip_b200 import _lib

    L = _lib.lib()
    buf = (ctypes.c_float * 64)()
    other = (ctypes.c_float * 64)()
    p, q = ctypes.addressof(buf), ctypes.addressof(other)
    assert L.cwx_add_rms_norm(None, p, None, p, EPS, 1, 64, p, q, None) == _lib.EINVAL
    assert L.cwx_add_rms_norm(p, p, None, p, EPS, -1, 64, p, q, None) == _lib.EINVAL
    assert L.cwx_add_rms_norm(p, p, None, p, EPS, 1, 0, p, q, None) == _lib.EINVAL
    assert L.cwx_add_rms_norm(p, q, None, p, EPS, 1, 64, p, q, None) == _lib.EINVAL  # out aliases b
    assert b"buffer of its own" in L.cwx_last_error()
    assert L.cwx_add_rms_norm(p, q, None, p, EPS, 0, 64, p, ctypes.addressof((ctypes.c_float * 64)()), None) == 0


# ---------------------------------------------------------------- GPU


def _gpu_add_norm(a, b, c, alpha, eps, offset=0):
    """The C-ABI call on device copies; offset > 0 places every row buffer `offset` floats into
    its allocation (unaligned rows: the scalar form of the kernel)."""
    import torch

    from coachwhip_b200 import _lib

    def dev(x):
        if x is None:
            return None, None
        base = torch.zeros(x.size + offset, dtype=torch.float32, device="cuda:0")
        view = base[offset:]
        view.copy_(torch.from_numpy(np.ascontiguousarray(x).reshape(-1)))
        return base, view

    keep = [dev(a), dev(b), dev(c), dev(alpha)]
    rows, H = a.shape
    s = torch.empty(rows * H + offset, dtype=torch.float32, device="cuda:0")[offset:]
    o = torch.empty(rows * H + offset, dtype=torch.float32, device="cuda:0")[offset:]
    ptr = [None if v is None else v.data_ptr() for _, v in keep]
    rc = _lib.lib().cwx_add_rms_norm(ptr[0], ptr[1], ptr[2], ptr[3], eps, rows, H, s.data_ptr(), o.data_ptr(), None)
    _lib.check(rc)
    torch.cuda.synchronize()
    return s.cpu().numpy().reshape(rows, H), o.cpu().numpy().reshape(rows, H)


def _check_norm(o, s, alpha, ref_o):
    err = np.abs(o.astype(np.float64) - ref_o.astype(np.float64))
    assert (err <= NORM_RTOL * np.abs(ref_o) + 1e-30).all(), f"max rel {np.max(err / (np.abs(ref_o) + 1e-30)):.3e}"
    ex = _exact(s, alpha, EPS)
    ulp = np.spacing(np.abs(ex).astype(np.float32)).astype(np.float64)
    assert (np.abs(o - ex) <= 8 * ulp + 1e-38).all()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,H,with_c", [(1, 2048, True), (64, 2048, True), (7, 2880, True), (5, 37, True),
                                           (3, 2048, False), (300, 512, True)])
def test_add_norm_matches_oracle(rows, H, with_c):
    a, b, c, alpha = _inputs(rows, H, rows * 7 + H, with_c)
    s, o = _gpu_add_norm(a, b, c, alpha, EPS)
    rs, ro = O.add_rms_norm(a, b, c, alpha, EPS)
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32))
    _check_norm(o, s, alpha, ro)


@pytest.mark.gpu
def test_add_norm_unaligned_rows_give_the_same_bits():
    a, b, c, alpha = _inputs(9, 2048, 5)
    s0, o0 = _gpu_add_norm(a, b, c, alpha, EPS)
    s1, o1 = _gpu_add_norm(a, b, c, alpha, EPS, offset=1)
    assert np.array_equal(s0.view(np.uint32), s1.view(np.uint32))
    assert np.array_equal(o0.view(np.uint32), o1.view(np.uint32))


@pytest.mark.gpu
def test_add_norm_edge_rows():
    # an all-zero row (out 0), a row whose squares overflow f32 (the reference's sum is inf:
    # out 0), tiny values near the f32 subnormal range, and a single huge element
    H = 256
    a = np.zeros((4, H), dtype=np.float32)
    a[1] = 3e19
    a[2] = np.float32(1e-20) * np.arange(1, H + 1, dtype=np.float32)
    a[3, 17] = 1e30
    b = np.zeros_like(a)
    alpha = np.full(H, 0.5, dtype=np.float32)
    s, o = _gpu_add_norm(a, b, None, alpha, EPS)
    rs, ro = O.add_rms_norm(a, b, None, alpha, EPS)
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(o[0], ro[0]) and np.array_equal(o[1], ro[1])  # zeros
    assert np.allclose(o[2:], ro[2:], rtol=NORM_RTOL, atol=0)


@pytest.mark.gpu
def test_add_norm_in_place_and_torch_mirror():
    import torch

    from coachwhip_b200.moe import add_norm

    a, b, c, alpha = _inputs(16, 1024, 3)
    ta, tb, tc, tw = (torch.from_numpy(v).to("cuda:0") for v in (a, b, c, alpha))
    s, o = add_norm(ta, tb, tc, tw, EPS)
    rs, ro = O.add_rms_norm(a, b, c, alpha, EPS)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    _check_norm(o.cpu().numpy(), rs, alpha, ro)
    with pytest.raises(ValueError, match="f32 only"):
        add_norm(ta.half(), tb, tc, tw, EPS)
    # in place: the sum written over a
    from coachwhip_b200 import _lib

    o2 = torch.empty_like(ta)
    _lib.check(_lib.lib().cwx_add_rms_norm(ta.data_ptr(), tb.data_ptr(), tc.data_ptr(), tw.data_ptr(), EPS, 16, 1024,
                                           ta.data_ptr(), o2.data_ptr(), None))
    assert torch.equal(ta, s) and torch.equal(o2, o)


SPEC = Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_S, up_type=O.IQ2_S, down_type=O.IQ3_S,
            shared_inter=256, seed=2)


@pytest.mark.gpu
@pytest.mark.parametrize("T,min_pile,mode", [(8, 0, O.MODE_CANDLE), (256, 1, O.MODE_F32)])
def test_fused_norm_in_moe_forward(T, min_pile, mode):
    import torch

    from coachwhip_b200 import _lib

    _lib.set_mma_min_pile(0, min_pile)
    try:
        L = build_cpu(SPEC)
        x = make_input(SPEC, T)
        rng = np.random.default_rng(T)
        res = rng.standard_normal((T, SPEC.hidden), dtype=np.float32)
        alpha = (1.0 + 0.1 * rng.standard_normal(SPEC.hidden)).astype(np.float32)
        moe = build_gpu(L, device=0, act_mode=mode)
        tx = torch.from_numpy(x).to("cuda:0")[None]
        tr = torch.from_numpy(res).to("cuda:0")[None]
        tw = torch.from_numpy(alpha).to("cuda:0")
        plain = moe.forward(tx, residual=tr)[0]
        out, normed = moe.forward_norm(tx, tr, tw, EPS)
        _lib.status(0)
        out, normed = out[0], normed[0]
        assert torch.equal(out, plain), "fused combine changed the layer output"
        # the standalone call on the layer's own output: the same bits
        _, o2 = _gpu_add_norm(out.cpu().numpy(), np.zeros((T, SPEC.hidden), np.float32), None, alpha, EPS)
        assert np.array_equal(normed.cpu().numpy().view(np.uint32), o2.view(np.uint32))
        # against the oracle's whole layer and residual step
        ref = O.moe_forward(L, x, mode)
        _, ro = O.add_rms_norm(ref["routed"], ref["shared"], res, alpha, EPS)
        assert rel_l2(normed.cpu().numpy(), ro) < 1e-3
        with pytest.raises(_lib.CwxError, match="buffer of its own"):
            A = _lib.MoeArgs()
            A.x, A.tokens, A.out = tx.data_ptr(), T, out.data_ptr()
            A.norm_w, A.norm_out = tw.data_ptr(), out.data_ptr()
            _lib.check(_lib.lib().cwx_moe_forward(_lib.ctx(0), ctypes.byref(moe._layer), ctypes.byref(A), None))
    finally:
        _lib.set_mma_min_pile(0, 32)
