"""Expert parallelism on the GPU through cwx_ep_dispatch / cwx_ep_experts / cwx_ep_combine.

Two ranks emulated in one process on one device (the exchanges are tensor copies between the
two engines), and the real two-process NCCL run when two devices are present. Same bar as the
single-device layer: expert ids bit-exact (through the routing), outputs within relative L2 1e-3
of the oracle."""

import os

import numpy as np
import pytest

import oracle as O
from tests.ep_common import gpu_engine, run_emulated
from tests.layers import Spec, build_cpu, make_input, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-3
SPECS = {
    "iq_mix": Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_S, up_type=O.IQ2_S,
                   down_type=O.IQ3_S, shared_inter=256, seed=2),
    "mxfp4_gptoss": Spec(hidden=576, n_experts=16, top_k=4, inter=576, gate_type=O.MXFP4, up_type=O.MXFP4,
                         down_type=O.MXFP4, act=O.ACT_CLAMPED_SWIGLU, router_bias=True, expert_bias=True, seed=4),
    "q4k": Spec(hidden=256, n_experts=8, top_k=2, inter=256, gate_type=O.Q4_K, up_type=O.Q4_K, down_type=O.Q4_K,
                shared_inter=256, seed=11),
}


def _emulated(L, x, world, mode):
    """All ranks' steps on device 0, exchanging by slicing; returns the concatenated outputs."""
    return run_emulated([gpu_engine(L, world, r, 0, mode) for r in range(world)], x)


@pytest.mark.parametrize("name,T,world", [("iq_mix", 64, 2), ("iq_mix", 512, 4), ("mxfp4_gptoss", 64, 2),
                                          ("q4k", 24, 2), ("q4k", 8, 1)])
@pytest.mark.parametrize("mode", [O.MODE_CANDLE, O.MODE_F32])
def test_ep_emulated_ranks_match_oracle(name, T, world, mode):
    s = SPECS[name]
    L = build_cpu(s)
    x = make_input(s, T)
    out = _emulated(L, x, world, mode)
    err = rel_l2(out, O.moe_forward(L, x, mode)["out"])
    assert err < RTOL, err


@pytest.mark.parametrize("name,T,world", [("iq_mix", 256, 4), ("mxfp4_gptoss", 64, 2), ("q4k", 24, 2)])
def test_ep_emulated_ranks_under_a_placement(name, T, world):
    # experts placed by a balanced placement of skewed counts (not contiguous ranges): each rank's
    # banks and bias rows hold the experts the placement gives it, in slot order
    from coachwhip_b200.ep import balanced_placement

    s = SPECS[name]
    L = build_cpu(s)
    x = make_input(s, T)
    counts = np.random.default_rng(5).zipf(1.5, s.n_experts).astype(np.float64)
    place = balanced_placement(counts, world)
    assert not np.array_equal(place, np.arange(s.n_experts))
    for mode in (O.MODE_CANDLE, O.MODE_F32):
        out = run_emulated([gpu_engine(L, world, r, 0, mode, placement=place) for r in range(world)], x)
        err = rel_l2(out, O.moe_forward(L, x, mode)["out"])
        assert err < RTOL, (mode, err)


def test_ep_rank_with_no_tokens_and_no_picks():
    # every token routes to rank 0's experts: rank 1 receives nothing, and sends nothing back
    s = SPECS["q4k"]
    L = build_cpu(s)
    L["router_b"] = np.zeros(8, dtype=np.float32)
    L["router_b"][1] = 50.0
    L["router_b"][2] = 49.0
    x = make_input(s, 16)
    out = _emulated(L, x, 2, O.MODE_F32)
    assert rel_l2(out, O.moe_forward(L, x, O.MODE_F32)["out"]) < RTOL


def test_ep_inconsistent_counts_are_refused():
    # a receive-count list that does not add up to the rows and records handed over
    import ctypes

    from coachwhip_b200 import CwxError, _lib

    s = SPECS["q4k"]
    L = build_cpu(s)
    eng = gpu_engine(L, 2, 0, 0, O.MODE_F32)
    rows = torch.zeros((3, s.hidden), dtype=eng.row_dtype, device="cuda")
    picks = torch.zeros((4, 3), dtype=torch.int32, device="cuda")
    with pytest.raises(CwxError, match="do not add up"):
        eng.experts(rows, picks, [1, 1], [2, 2])
    _lib.status(0)


def _nccl_rank(rank, world, port, q):
    import torch.distributed as dist

    from coachwhip_b200.ep import ExpertParallelMoe

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        s = SPECS["iq_mix"]
        L = build_cpu(s)
        T = 256
        x = make_input(s, T)
        per = T // world
        moe = ExpertParallelMoe(gpu_engine(L, world, rank, rank, O.MODE_F32))
        xl = torch.from_numpy(np.ascontiguousarray(x[rank * per:(rank + 1) * per])).cuda(rank)
        out = moe.forward(xl[None])[0].cpu().numpy()
        want = O.moe_forward(L, x, O.MODE_F32)["out"][rank * per:(rank + 1) * per]
        q.put((rank, rel_l2(out, want)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two devices")
def test_ep_nccl_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_nccl_rank, args=(r, 2, 29641, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) < RTOL, res


# ---------------------------------------------------------------- the library's own transport
@pytest.mark.parametrize("name", ["iq_mix", "mxfp4_gptoss", "q4k"])
@pytest.mark.parametrize("mode", [O.MODE_F32, O.MODE_CANDLE])
def test_ep_forward_one_rank_matches_oracle(name, mode):
    # cwx_ep_forward on a one-rank NCCL communicator: the whole layer (dispatch, both fixed-capacity
    # exchanges, experts, combine) in one call, with a capacity above the tokens so the segments
    # have unused rows
    from coachwhip_b200 import _lib
    from coachwhip_b200.ep import EpComm, LibraryExpertParallelMoe

    s = SPECS[name]
    L = build_cpu(s)
    T = 96
    x = make_input(s, T)
    comm = EpComm(0, 1, 0, share=lambda b: b)
    moe = LibraryExpertParallelMoe(gpu_engine(L, 1, 0, 0, mode), comm, T + 37)
    taps = {}
    out = moe.forward(torch.from_numpy(x).cuda()[None], taps=taps)[0].cpu().numpy()
    _lib.status(0)
    ref = O.moe_forward(L, x, mode)
    assert np.array_equal(taps["ids"].cpu().numpy().astype(np.uint32), ref["ids"])
    assert rel_l2(out, ref["out"]) < RTOL
    # a second call with fewer tokens reuses the buffers; nothing of the first call shows through
    out2 = moe.forward(torch.from_numpy(x[:40]).cuda()[None])[0].cpu().numpy()
    _lib.status(0)
    assert rel_l2(out2, O.moe_forward(L, x[:40], mode)["out"]) < RTOL
    comm.close()


def test_ep_forward_refuses_tokens_above_capacity():
    import ctypes

    from coachwhip_b200 import CwxError, _lib
    from coachwhip_b200.ep import EpComm

    s = SPECS["q4k"]
    L = build_cpu(s)
    eng = gpu_engine(L, 1, 0, 0, O.MODE_F32)
    comm = EpComm(0, 1, 0, share=lambda b: b)
    x = torch.zeros((8, s.hidden), device="cuda")
    out = torch.empty_like(x)
    with pytest.raises(CwxError, match="capacity"):
        _lib.check(_lib.lib().cwx_ep_forward(_lib.ctx(0), comm.handle, ctypes.byref(eng._layer),
                                             ctypes.byref(eng._group), x.data_ptr(), 8, 4, None, out.data_ptr(),
                                             None, None))
    comm.close()


def _lib_rank(rank, world, port, q):
    import torch.distributed as dist

    from coachwhip_b200 import _lib
    from coachwhip_b200.ep import EpComm, LibraryExpertParallelMoe

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        s = SPECS["iq_mix"]
        L = build_cpu(s)
        x = make_input(s, 228)
        lo, hi = (0, 128) if rank == 0 else (128, 228)  # uneven token counts, capacity 128
        comm = EpComm(rank, world, rank)
        moe = LibraryExpertParallelMoe(gpu_engine(L, world, rank, rank, O.MODE_F32), comm, 128)
        xl = torch.from_numpy(np.ascontiguousarray(x[lo:hi])).cuda(rank)
        out = moe.forward(xl[None])[0].cpu().numpy()
        _lib.status(rank)
        want = O.moe_forward(L, x, O.MODE_F32)["out"][lo:hi]
        q.put((rank, rel_l2(out, want)))
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two devices")
def test_ep_forward_two_ranks_nccl():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_lib_rank, args=(r, 2, 29643, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) < RTOL, res
