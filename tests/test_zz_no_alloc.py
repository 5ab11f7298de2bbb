"""cwx_permute_noalloc (fixed device scratch, no allocation) against cwx_permute.

Named to be collected last, so it also runs after every other GPU test has used the library."""

import numpy as np
import pytest

from coachwhip_b200 import CwxError, _lib


def _noalloc(ids, T, K, E, pairs, heads, status=None, stream=None):
    return _lib.lib().cwx_permute_noalloc(ids, T, K, E, pairs, heads, status, stream)


def test_oversize_is_refused_before_device_work():
    # the size checks come before any CUDA call, so this runs without a GPU
    # (the non-null placeholder pointers are never dereferenced: the call is refused first)
    rc = _noalloc(16, 1 << 20, 8, 512, 16, 16)
    assert rc == _lib.EINVAL
    assert "scratch words" in _lib.lib().cwx_last_error().decode()
    assert _noalloc(16, 1, 1, 5000, 16, 16) == _lib.EINVAL
    assert "n_experts" in _lib.lib().cwx_last_error().decode()


def _case(T, K, E, seed):
    import torch

    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    return torch.from_numpy(ids).cuda()


@pytest.mark.gpu
def test_two_calls_in_a_row_match_cwx_permute():
    import torch

    from coachwhip_b200.moe import piles

    # a large call, then a smaller one with fewer experts: stale scratch from the first call
    # would show in the second
    cases = [(4096, 8, 256, 1), (37, 10, 64, 2)]
    outs = []
    st = torch.cuda.current_stream().cuda_stream
    for T, K, E, seed in cases:
        ids = _case(T, K, E, seed)
        pairs = torch.full((T * K,), -1, dtype=torch.int32, device="cuda")
        heads = torch.full((E, 3), -1, dtype=torch.int32, device="cuda")
        status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
        _lib.check(_noalloc(ids.data_ptr(), T, K, E, pairs.data_ptr(), heads.data_ptr(), status.data_ptr(), st))
        outs.append((ids, pairs, heads, status))
    torch.cuda.synchronize()
    for (T, K, E, _), (ids, pairs, heads, status) in zip(cases, outs):
        want_p, want_h = piles(ids, E)
        assert torch.equal(pairs, want_p)
        assert torch.equal(heads, want_h)
        assert int(status.item()) == 0


@pytest.mark.gpu
def test_bad_id_sets_status_and_next_call_clears_it():
    import torch

    st = torch.cuda.current_stream().cuda_stream
    ids = torch.tensor([[0, 9]], dtype=torch.int32, device="cuda")
    pairs = torch.empty(2, dtype=torch.int32, device="cuda")
    heads = torch.empty((4, 3), dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_noalloc(ids.data_ptr(), 1, 2, 4, pairs.data_ptr(), heads.data_ptr(), status.data_ptr(), st))
    torch.cuda.synchronize()
    assert int(status.item()) != 0
    ids = torch.tensor([[0, 3]], dtype=torch.int32, device="cuda")
    _lib.check(_noalloc(ids.data_ptr(), 1, 2, 4, pairs.data_ptr(), heads.data_ptr(), status.data_ptr(), st))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert pairs.tolist() == [0, 1]
