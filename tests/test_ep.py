"""Expert parallelism, host side: the exchange protocol of ExpertParallelMoe on two gloo ranks
(CPU), with the per-rank steps computed by the oracle. Each rank's output must equal the
single-process layer's output for its tokens."""

import os

import numpy as np
import pytest

import oracle as O
from tests.layers import Spec, build_cpu, make_input, rel_l2

SPEC = Spec(hidden=256, n_experts=8, top_k=2, inter=256, gate_type=O.Q4_K, up_type=O.Q4_K, down_type=O.Q4_K,
            shared_inter=256, seed=11)
# the gpt-oss layer shape: MXFP4 experts with per-expert biases, clamped SwiGLU, router bias
SPEC_GPTOSS = Spec(hidden=256, n_experts=8, top_k=4, inter=256, gate_type=O.MXFP4, up_type=O.MXFP4,
                   down_type=O.MXFP4, act=O.ACT_CLAMPED_SWIGLU, router_bias=True, expert_bias=True, seed=12)
T = 24


def _rank(rank, world, port, q, spec=SPEC):
    import torch
    import torch.distributed as dist

    from coachwhip_b200.ep import ExpertParallelMoe
    from tests.ep_common import OracleEngine

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = build_cpu(spec)
        x = make_input(spec, T)
        per = T // world
        xl = torch.from_numpy(np.ascontiguousarray(x[rank * per:(rank + 1) * per]))
        moe = ExpertParallelMoe(OracleEngine(L, world, rank, O.MODE_F32))
        out = moe.forward(xl[None])[0].numpy()
        want = O.moe_forward(L, x, O.MODE_F32)["out"][rank * per:(rank + 1) * per]
        q.put((rank, rel_l2(out, want)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("spec,port", [(SPEC, 29611), (SPEC_GPTOSS, 29613)], ids=["qwen", "gptoss"])
def test_expert_parallel_protocol_on_two_gloo_ranks(spec, port):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q, spec)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) < 1e-5, res


def _rank_dies(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    from coachwhip_b200.ep import ExpertParallelMoe
    from tests.ep_common import OracleEngine

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    if rank == 1:
        os._exit(0)  # the peer dies between layers, with nothing in flight
    L = build_cpu(SPEC)
    x = torch.from_numpy(np.ascontiguousarray(make_input(SPEC, T)[: T // world]))
    moe = ExpertParallelMoe(OracleEngine(L, world, rank, O.MODE_F32))
    try:
        moe.forward(x[None])
        q.put("completed")
    except Exception as e:  # the exchange reports the lost peer instead of waiting forever
        q.put(f"raised: {type(e).__name__}")


def test_lost_peer_is_reported_not_waited_on():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_dies, args=(r, 2, 29613, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    alive = [p.is_alive() for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert not any(alive)
    msg = q.get(timeout=5)
    assert msg.startswith("raised"), msg


def test_balanced_placement():
    # a permutation of the expert slots, equal experts per rank, and on skewed counts the busiest
    # rank's load at most the mean plus the largest single count (the greedy bound)
    from coachwhip_b200.ep import balanced_placement, expert_lists

    rng = np.random.default_rng(0)
    for E, W in ((16, 2), (512, 4), (512, 8), (8, 1)):
        c = rng.zipf(1.3, E).astype(np.float64)
        s = balanced_placement(c, W)
        assert sorted(s.tolist()) == list(range(E))
        lists = expert_lists(s, W)
        assert [len(x) for x in lists] == [E // W] * W
        for r, x in enumerate(lists):
            assert [int(s[e]) for e in x] == [r * (E // W) + i for i in range(E // W)]
        load = np.array([c[x].sum() for x in lists])
        assert load.max() <= load.mean() + c.max() + 1e-9
    with pytest.raises(ValueError):
        balanced_placement(np.ones(10), 4)
