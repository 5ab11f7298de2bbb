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


def _run(T, K, E, seed, st):
    import torch

    ids = _case(T, K, E, seed)
    pairs = torch.full((T * K,), -1, dtype=torch.int32, device="cuda")
    heads = torch.full((E, 3), -1, dtype=torch.int32, device="cuda")
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    _lib.check(_noalloc(ids.data_ptr(), T, K, E, pairs.data_ptr(), heads.data_ptr(), status.data_ptr(), st))
    return ids, pairs, heads, status


def _check(E, ids, pairs, heads, status):
    import torch

    from coachwhip_b200.moe import piles

    want_p, want_h = piles(ids, E)
    assert torch.equal(pairs, want_p)
    assert torch.equal(heads, want_h)
    assert int(status.item()) == 0


@pytest.mark.gpu
def test_two_calls_in_a_row_match_cwx_permute():
    import torch

    # every call takes the three-kernel path (more than 2048 picks), whose per-tile counts live in
    # the shared array: a large call, a smaller one with fewer experts and tiles (the first call's
    # counts would show through if a region were not rewritten), then the first size again
    cases = [(4096, 8, 256, 1), (3000, 8, 64, 2), (4096, 8, 256, 3)]
    st = torch.cuda.current_stream().cuda_stream
    outs = [_run(T, K, E, seed, st) for T, K, E, seed in cases]
    torch.cuda.synchronize()
    for (T, K, E, _), out in zip(cases, outs):
        _check(E, *out)


@pytest.mark.gpu
def test_largest_accepted_size_matches_cwx_permute():
    import torch

    # 214 tiles x 1208 experts + 3 x 1208 + 8 = 262,144 words: exactly the array; one pick more
    # needs another tile and is refused
    T, K, E = 27392, 8, 1208
    assert (T * K + 1023) // 1024 * E + 3 * E + 8 == _lib.NOALLOC_SCRATCH_WORDS
    st = torch.cuda.current_stream().cuda_stream
    out = _run(T, K, E, 4, st)
    torch.cuda.synchronize()
    _check(E, *out)
    assert _noalloc(16, T * K + 1, 1, E, 16, 16) == _lib.EINVAL


@pytest.mark.gpu
def test_calls_leave_device_memory_unchanged():
    import torch

    # after a first call of the same shape (which looks up the array's address and loads the
    # kernels), further calls take no device memory
    st = torch.cuda.current_stream().cuda_stream
    T, K, E = 5000, 8, 256
    ids = _case(T, K, E, 5)
    pairs = torch.empty(T * K, dtype=torch.int32, device="cuda")
    heads = torch.empty((E, 3), dtype=torch.int32, device="cuda")
    _lib.check(_noalloc(ids.data_ptr(), T, K, E, pairs.data_ptr(), heads.data_ptr(), None, st))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _lib.check(_noalloc(ids.data_ptr(), T, K, E, pairs.data_ptr(), heads.data_ptr(), None, st))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    _check(E, ids, pairs, heads, torch.zeros(1, dtype=torch.int32, device="cuda"))


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
