"""Benchmark: coachwhip's MoE layer on B200.

Workload (`config.workload`): the Qwen3.6-35B-A3B-shaped decode stack, 40 MoE layers with every
expert resident in HBM: hidden 2048, 256 routed experts, top-8 renormalised, intermediate 512,
gate/up IQ2_S and down IQ3_S from N(0, 0.02) (seed 2), one Q4_K shared expert with a sigmoid
gate, router f32. A step is one pass of a batch of tokens through the 40 layers
(x <- x + moe_l(x)); the headline batch is 64 tokens, and the sweep reports 1, 4, 16, 64.
Synthetic data: weights and inputs come from the library's seeded generator (no model file).

value:   tokens/s with inputs resident in HBM, the 40-layer stack replayed as one CUDA graph.
e2e:     tokens/s through the public API (StreamedMoe.forward per layer) including the pinned
         host->device copy of the step's tokens and the device->host read of the result.
roofline: the expert-product kernel (k_gemv), algorithmic bytes (quantised weight bytes of the
         experts each launch reads + activation traffic) over its CUDA-event duration, against
         the measured HBM copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline: the CPU restatement of the reference's layer (oracle/, candle semantics) timed on
         the host cores on one full layer of the same bank at the same batch.
prefill: config 2 (the config-1 layers at 1500 and 4096 tokens, tensor-core products).
config3: the gpt-oss-shaped stack (36 MXFP4 layers): decode 1 and 64 and prefill of 4096 tokens
         on one GPU; on N ranks the 4096-token prefill expert-parallel.
expert_parallel (N > 1): config 4 (48 layers, 512 experts, 8192 tokens) expert-parallel.

usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cwx|reference] [--batch T]
                       [--no-sweep] [--no-prefill] [--no-ep] [--no-c3] [--no-cpu] [--c3-layers L]
                       [--prefill-tokens T ...]
For N > 1 it runs under torchrun: config 1 does not shard (one process per GPU runs its own
replica; scaling "weak"); configs 3 and 4 shard their experts over the ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, E, K, I, I_S, LAYERS, SEED = 2048, 256, 8, 512, 512, 40, 2
T_GATE, T_UP, T_DOWN, T_RW, T_SG, T_SU, T_SD, T_SGI, T_IN = 0, 1, 2, 3, 5, 6, 7, 8, 12
METRIC = "MoE-layer tokens/s (decode b=1-64, prefill 4K) and % of HBM/tensor roofline"
WORKLOAD = "config1 decode stack: 40 x MoE(H2048, E256, top8, I512, IQ2_S gate/up, IQ3_S down, Q4_K shared)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="cwx", choices=["cwx", "reference"])
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--layers", type=int, default=LAYERS)
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-prefill", action="store_true")
    p.add_argument("--no-ep", action="store_true")
    p.add_argument("--no-c3", action="store_true", help="skip the config-3 (MXFP4, gpt-oss shape) runs")
    p.add_argument("--c3-layers", type=int, default=C3_LAYERS, help="config-3 layers (36; fewer for profiling)")
    p.add_argument("--prefill-tokens", type=int, nargs="*", default=None,
                   help="config-2 prefill sizes (default 1500 4096; one size for profiling)")
    return p.parse_args()


def dist_setup():
    import torch

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    return rank, world, local


def stream(seed, layer, tensor):
    """cwx_stream(): the per-tensor key of the seeded generator (synth_math.h)."""
    def sm(x):
        x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return x ^ (x >> 31)

    return sm((seed << 40) ^ (layer << 16) ^ tensor)


def synth_f32(n, key, std, dev):
    import torch

    from coachwhip_b200 import _lib

    out = torch.empty(n, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().cwx_synth_normal(_lib.ctx(dev.index), key, 0, n, std, out.data_ptr(),
                                           torch.cuda.current_stream(dev).cuda_stream))
    return out


def build_stack(dev, layers):
    from coachwhip_b200 import TYPE_IQ2_S, TYPE_IQ3_S, TYPE_Q4_K
    from coachwhip_b200.moe import Bank, ExpertAct, ExpertStore, SharedExpert, StreamedMoe

    d = dev.index
    banks, mods = [], []
    for l in range(layers):
        g = Bank.synth(TYPE_IQ2_S, I, H, E, stream(SEED, l, T_GATE), 0.02, d)
        u = Bank.synth(TYPE_IQ2_S, I, H, E, stream(SEED, l, T_UP), 0.02, d)
        dn = Bank.synth(TYPE_IQ3_S, H, I, E, stream(SEED, l, T_DOWN), 0.02, d)
        banks.append((g, u, dn))
    store = ExpertStore(banks)
    for l in range(layers):
        sh = SharedExpert(synth_f32(H, stream(SEED, l, T_SGI), 0.02, dev),
                          Bank.synth(TYPE_Q4_K, I_S, H, 1, stream(SEED, l, T_SG), 0.02, d),
                          Bank.synth(TYPE_Q4_K, I_S, H, 1, stream(SEED, l, T_SU), 0.02, d),
                          Bank.synth(TYPE_Q4_K, H, I_S, 1, stream(SEED, l, T_SD), 0.02, d))
        w = synth_f32(E * H, stream(SEED, l, T_RW), 0.02, dev).view(E, H)
        mods.append(StreamedMoe(l, w, K, True, ExpertAct.Silu(), store, shared=sh))
    return store, mods


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def run_stack(mods, x):
    h = x
    for m in mods:
        h = m.forward(h, residual=h)
    return h


def time_graph(graph, steps, warmup, dev):
    import torch

    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / steps


def capture(mods, x, dev):
    import torch

    run_stack(mods, x)  # warm the kernels outside capture
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            out = run_stack(mods, x)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    return g, out


def used_experts(mods, x):
    """Unique experts each layer routes to for this batch (from the routing taps)."""
    import torch

    us = []
    h = x
    for m in mods:
        taps = {}
        h2 = m.forward(h, residual=h, taps=taps)
        us.append(int(torch.unique(taps["ids"]).numel()))
        h = h2
    return us


def oracle_layer(bank_bytes=None):
    """One config-1 layer for the CPU oracle (layer 0; bank bytes from the GPU when given)."""
    import oracle as O

    L = dict(hidden=H, n_experts=E, top_k=K, inter=I, norm_topk_prob=1, gate_type=O.IQ2_S, up_type=O.IQ2_S,
             down_type=O.IQ3_S, act=O.ACT_SILU, shared_inter=I_S, sh_gate_type=O.Q4_K, sh_up_type=O.Q4_K,
             sh_down_type=O.Q4_K)
    if bank_bytes is None:
        L["gate_bank"] = O.synth_matrix(O.IQ2_S, stream(SEED, 0, T_GATE), 0, E, I, H, 0.02)
        L["up_bank"] = O.synth_matrix(O.IQ2_S, stream(SEED, 0, T_UP), 0, E, I, H, 0.02)
        L["down_bank"] = O.synth_matrix(O.IQ3_S, stream(SEED, 0, T_DOWN), 0, E, H, I, 0.02)
    else:
        L["gate_bank"], L["up_bank"], L["down_bank"] = bank_bytes
    L["router_w"] = O.normal(stream(SEED, 0, T_RW), 0, E * H, 0.02).reshape(E, H)
    L["sh_gate"] = O.synth_matrix(O.Q4_K, stream(SEED, 0, T_SG), 0, 1, I_S, H, 0.02)
    L["sh_up"] = O.synth_matrix(O.Q4_K, stream(SEED, 0, T_SU), 0, 1, I_S, H, 0.02)
    L["sh_down"] = O.synth_matrix(O.Q4_K, stream(SEED, 0, T_SD), 0, 1, H, I_S, 0.02)
    L["sh_gate_inp"] = O.normal(stream(SEED, 0, T_SGI), 0, H, 0.02)
    return L


def cpu_baseline(store, T, budget_s=12.0):
    """The oracle (CPU restatement of the reference's layer) on layer 0 of the same bank."""
    import oracle as O

    g, u, d = store.banks[0]
    L = oracle_layer((g.download(), u.download(), d.download()))
    x = O.normal(stream(SEED, 0, T_IN), 0, T * H, 1.0).reshape(T, H)
    O.moe_forward(L, x, O.MODE_CANDLE)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        O.moe_forward(L, x, O.MODE_CANDLE)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 50:
            break
    per_layer = el / n
    return {"value": T / (per_layer * LAYERS), "unit": "tokens/s", "cores": O.get_threads(), "kind": "port",
            "sample": f"{n} calls of one full config-1 layer (256 experts, batch {T}) through the C++ restatement "
                      f"of the reference (oracle/) on the host; tokens/s = batch / (40 x per-layer time)",
            "per_layer_ms": per_layer * 1e3}


def impl_reference(a, rank, world):
    if rank != 0:
        return
    import oracle as O

    T = a.batch
    L = oracle_layer()
    x = O.normal(stream(SEED, 0, T_IN), 0, T * H, 1.0).reshape(T, H)
    for _ in range(a.warmup):
        O.moe_forward(L, x, O.MODE_CANDLE)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        O.moe_forward(L, x, O.MODE_CANDLE)  # one layer per step: a bounded sample of the stack
    per_layer = (time.perf_counter() - t0) / a.steps
    v = T / (per_layer * LAYERS)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": per_layer * 1e3 * LAYERS,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": T, "layers": LAYERS, "sample": "one layer per step, x40"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": O.get_threads(), "kind": "port",
                             "sample": f"each step: one full config-1 layer (256 experts, batch {T}) on the host "
                                       f"CPU through the C++ restatement of the reference (oracle/); tokens/s = "
                                       f"batch / (40 x per-layer time)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PREFILL_T = [1500, 4096]

# Config 4 (expert parallelism, measured when the bench runs on 2+ ranks): 48 layers of
# H2048 / E512 / top-10 / I512, IQ3_S gate/up, Q4_K down, a Q4_K shared expert, Zipf(1.1) router
# bias over a seeded permutation of the experts, 8192 tokens split evenly over the ranks.
EP_H, EP_E, EP_K, EP_I, EP_IS, EP_LAYERS, EP_SEED, EP_T = 2048, 512, 10, 512, 512, 48, 5, 8192


def ep_runs(world, rank, local, a, maxall, barrier):
    import numpy as np
    import torch

    from coachwhip_b200 import TYPE_IQ3_S, TYPE_Q4_K, _lib
    from coachwhip_b200.ep import CudaEngine, ExpertParallelMoe
    from coachwhip_b200.moe import Bank, ExpertAct, SharedExpert

    dev = torch.device(f"cuda:{local}")
    epr = EP_E // world
    r = np.random.default_rng(EP_SEED).permutation(EP_E) + 1
    zb = (-1.1 * np.log(r) - np.log(np.sum(np.arange(1, EP_E + 1, dtype=np.float64) ** -1.1))).astype(np.float32)
    zipf = torch.from_numpy(zb).to(dev)
    layers = []
    for l in range(EP_LAYERS):
        g = Bank.synth(TYPE_IQ3_S, EP_I, EP_H, epr, stream(EP_SEED, l, T_GATE), 0.02, local, first=rank * epr)
        u = Bank.synth(TYPE_IQ3_S, EP_I, EP_H, epr, stream(EP_SEED, l, T_UP), 0.02, local, first=rank * epr)
        d = Bank.synth(TYPE_Q4_K, EP_H, EP_I, epr, stream(EP_SEED, l, T_DOWN), 0.02, local, first=rank * epr)
        sh = SharedExpert(synth_f32(EP_H, stream(EP_SEED, l, T_SGI), 0.02, dev),
                          Bank.synth(TYPE_Q4_K, EP_IS, EP_H, 1, stream(EP_SEED, l, T_SG), 0.02, local),
                          Bank.synth(TYPE_Q4_K, EP_IS, EP_H, 1, stream(EP_SEED, l, T_SU), 0.02, local),
                          Bank.synth(TYPE_Q4_K, EP_H, EP_IS, 1, stream(EP_SEED, l, T_SD), 0.02, local))
        w = synth_f32(EP_E * EP_H, stream(EP_SEED, l, T_RW), 0.02, dev).view(EP_E, EP_H)
        eng = CudaEngine(w, EP_K, True, ExpertAct.Silu(), (g, u, d), world, rank, gate_bias=zipf, shared=sh,
                         act_mode=_lib.ACT_MODE_F32)
        eng._keep = (g, u, d, sh, w)
        layers.append(ExpertParallelMoe(eng))
    per = EP_T // world
    x = synth_f32(EP_T * EP_H, stream(EP_SEED + 1, 0, T_IN), 1.0, dev).view(EP_T, EP_H)[rank * per:(rank + 1) * per]
    x = x.contiguous().view(1, per, EP_H)

    def run():
        h = x
        for m in layers:
            h = m.forward(h, residual=h)
        return h

    for _ in range(max(1, a.warmup // 2)):
        run()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 2
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = maxall(e0.elapsed_time(e1) / reps)
    _lib.status(local)
    fl = EP_LAYERS * (2 * EP_T * EP_K * 3 * EP_H * EP_I + 2 * EP_T * 3 * EP_H * EP_IS + 2 * EP_T * EP_H * EP_E)
    return {"config": "config 4: 48 x MoE(H2048, E512, top10, I512, IQ3_S gate/up, Q4_K down, Q4_K shared, "
                      "Zipf(1.1) router bias)", "tokens": EP_T, "tokens_per_rank": per, "ranks": world,
            "experts_per_rank": epr, "ms_per_step": ms, "tokens_per_s": EP_T / (ms / 1e3),
            "tflops": fl / (ms / 1e3) / 1e12, "act_mode": "f32 activations (O2 semantics)",
            "transport": "NCCL all-to-all (torch.distributed all_to_all_single), one host read of the counts "
                         "per layer", "timing": f"CUDA events over {reps} eager passes of the 48 layers, max over ranks"}


# config 3: gpt-oss-120b-shaped MoE (MXFP4 experts with per-expert biases, clamped SwiGLU, router
# bias, top-4 renormalised, no shared expert)
C3_H, C3_E, C3_K, C3_I, C3_LAYERS, C3_SEED, C3_T = 2880, 128, 4, 2880, 36, 4, 4096
T_GB, T_UB, T_DB, T_RB = 9, 10, 11, 13


def c3_layers(world, rank, local, layers=C3_LAYERS):
    """This rank's config-3 layers: banks and biases of experts rank*epr .. (rank+1)*epr - 1."""
    from coachwhip_b200 import TYPE_MXFP4
    from coachwhip_b200.moe import Bank, ExpertAct

    import torch

    dev = torch.device(f"cuda:{local}")
    epr = C3_E // world
    out = []
    for l in range(layers):
        st = lambda t: stream(C3_SEED, l, t)  # noqa: E731
        g = Bank.synth(TYPE_MXFP4, C3_I, C3_H, epr, st(T_GATE), 0.02, local, first=rank * epr)
        u = Bank.synth(TYPE_MXFP4, C3_I, C3_H, epr, st(T_UP), 0.02, local, first=rank * epr)
        d = Bank.synth(TYPE_MXFP4, C3_H, C3_I, epr, st(T_DOWN), 0.02, local, first=rank * epr)
        gb = synth_f32(C3_E * C3_I, st(T_GB), 0.02, dev).view(C3_E, C3_I)[rank * epr:(rank + 1) * epr].contiguous()
        ub = synth_f32(C3_E * C3_I, st(T_UB), 0.02, dev).view(C3_E, C3_I)[rank * epr:(rank + 1) * epr].contiguous()
        db = synth_f32(C3_E * C3_H, st(T_DB), 0.02, dev).view(C3_E, C3_H)[rank * epr:(rank + 1) * epr].contiguous()
        w = synth_f32(C3_E * C3_H, st(T_RW), 0.02, dev).view(C3_E, C3_H)
        rb = synth_f32(C3_E, st(T_RB), 0.02, dev)
        out.append(((g, u, d), ExpertAct.ClampedSwiglu(1.702, 7.0, gb, ub, db), w, rb))
    return out


def c3_runs(world, rank, local, a, pk, maxall, barrier):
    """Config 3: decode batches 1 and 64 and prefill of 4096 tokens on one GPU (36-layer stack as
    CUDA graphs); on N ranks, the 4096-token prefill expert-parallel (128 / N experts per rank)."""
    import numpy as np
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200.moe import ExpertStore, StreamedMoe

    dev = torch.device(f"cuda:{local}")
    cfg = ("config 3: 36 x MoE(H2880, E128, top4, I2880, MXFP4 gate/up/down with per-expert biases, clamped "
           "SwiGLU 1.702/7.0, router bias, no shared expert); candle activation policy (Q8_0 codes)")
    t0 = time.time()
    layers = c3_layers(world, rank, local, a.c3_layers)
    torch.cuda.synchronize(dev)
    synth_s = time.time() - t0
    nl = len(layers)
    b_exp = 3 * C3_H * C3_I // 32 * 17 + (2 * C3_I + C3_H) * 4  # MXFP4 bytes of one expert + its biases
    if world > 1:
        from coachwhip_b200.ep import CudaEngine, ExpertParallelMoe

        mods = []
        for (banks, act, w, rb) in layers:
            eng = CudaEngine(w, C3_K, True, act, banks, world, rank, gate_bias=rb)
            eng._keep = (banks, act, w, rb)
            mods.append(ExpertParallelMoe(eng))
        per = C3_T // world
        x = synth_f32(C3_T * C3_H, stream(C3_SEED + 1, 0, T_IN), 1.0, dev).view(C3_T, C3_H)[rank * per:(rank + 1) * per]
        x = x.contiguous().view(1, per, C3_H)

        def run():
            h = x
            for m in mods:
                h = m.forward(h, residual=h)
            return h

        for _ in range(max(1, a.warmup // 2)):
            run()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 2
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = maxall(e0.elapsed_time(e1) / reps)
        _lib.status(local)
        fl = nl * (2 * C3_T * C3_K * 3 * C3_H * C3_I + 2 * C3_T * C3_H * C3_E)
        return {"config": cfg, "layers": nl, "prefill": {"tokens": C3_T, "tokens_per_rank": per, "ranks": world,
                                           "experts_per_rank": C3_E // world, "ms_per_step": ms,
                                           "tokens_per_s": C3_T / (ms / 1e3), "tflops": fl / (ms / 1e3) / 1e12,
                                           "timing": f"CUDA events over {reps} eager passes, max over ranks"},
                "bank_synthesis_s": synth_s}
    store = ExpertStore([b for (b, _, _, _) in layers])
    mods = [StreamedMoe(l, w, C3_K, True, act, store, gate_bias=rb) for l, (_, act, w, rb) in enumerate(layers)]
    for m in mods:
        m.reserve(C3_T)
    res = {"config": cfg, "layers": nl, "bank_gb": nl * C3_E * b_exp / 1e9, "bank_synthesis_s": synth_s, "decode": {}}
    for T in (1, 64):
        x = synth_f32(T * C3_H, stream(C3_SEED + 1, 0, T_IN), 1.0, dev).view(1, T, C3_H)
        g, _ = capture(mods, x, dev)
        ms = time_graph(g, max(5, a.steps // 2), a.warmup, dev)
        del g
        us = used_experts(mods, x)
        eb = sum(us) * b_exp + nl * C3_E * C3_H * 4  # experts read + router weights
        res["decode"][str(T)] = {"tokens_per_s": T / (ms / 1e3), "ms_per_step": ms,
                                 "unique_experts_mean": float(np.mean(us)),
                                 "hbm_gbs_expert_bytes": eb / (ms / 1e3) / 1e9,
                                 "hbm_frac": eb / (ms / 1e3) / 1e9 / pk["hbm_gbs"]}
        print(f"[bench] config 3 decode {T}: {ms:.3f} ms/step, {T / (ms / 1e3):.1f} tokens/s", file=sys.stderr,
              flush=True)
    x = synth_f32(C3_T * C3_H, stream(C3_SEED + 1, 0, T_IN), 1.0, dev).view(1, C3_T, C3_H)
    g, _ = capture(mods, x, dev)
    ms = time_graph(g, 3, max(1, a.warmup // 2), dev)
    del g
    fl = nl * (2 * C3_T * C3_K * 3 * C3_H * C3_I + 2 * C3_T * C3_H * C3_E)
    res["prefill"] = {"tokens": C3_T, "ms_per_step": ms, "tokens_per_s": C3_T / (ms / 1e3),
                      "tflops": fl / (ms / 1e3) / 1e12,
                      "path": "grouped mma.sync products (MXFP4 is not a tensor-core (tcgen05) format here)"}
    print(f"[bench] config 3 prefill {C3_T}: {ms:.3f} ms/step", file=sys.stderr, flush=True)
    _lib.status(local)
    return res


def layer_flops(T):
    """Multiply-add FLOPs of one config-1 layer on T tokens: routed gate/up/down, shared expert, router."""
    return 2 * T * K * 3 * H * I + 2 * T * 3 * H * I_S + 2 * T * H * E


def prefill_runs(mods, Ts, a, dev, pk, maxall, barrier, world):
    """Config 2: the 40-layer stack on 1500 and 4096 tokens (CUDA graphs), with the per-phase event
    times of one replay; the routed products run on the tensor-core kernel (k_mma)."""
    import torch

    from coachwhip_b200 import _lib

    out = {}
    ctx = _lib.ctx(dev.index)
    # the products run inside a long step: the sustained (power-capped) dense bf16 figure
    tpk = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    for T in Ts:
        x = synth_f32(T * H, stream(3, 0, T_IN), 1.0, dev).view(1, T, H)
        g, _ = capture(mods, x, dev)
        barrier()
        ms = maxall(time_graph(g, max(3, a.steps // 4), a.warmup, dev))
        del g
        _lib.lib().cwx_ctx_reset_profile(ctx)
        _lib.lib().cwx_ctx_set_profiling(ctx, 1)
        run_stack(mods, x)
        _lib.lib().cwx_ctx_set_profiling(ctx, 0)
        msv, _ = _lib.read_profile(dev.index)
        _lib.lib().cwx_ctx_reset_profile(ctx)
        ph = {n: msv[i] for i, n in enumerate(_lib.PHASES)}
        fl = len(mods) * layer_flops(T)
        prod_fl = len(mods) * (2 * T * K * 3 * H * I + 2 * T * 3 * H * I_S)
        prod_ms = ph["gate_up"] + ph["down"]
        out[str(T)] = {"tokens_per_s": world * T / (ms / 1e3), "ms_per_step": ms, "layers": len(mods),
                       "tflops": fl / (ms / 1e3) / 1e12, "frac_bf16_sustained_peak": fl / (ms / 1e3) / 1e12 / tpk,
                       "products_tflops": prod_fl / (prod_ms / 1e3) / 1e12, "phase_ms_eager": ph,
                       "act_mode": "f32 activations (O2 semantics)",
                       "path": "tcgen05 grouped products (k_mma) for the routed and shared experts, tiled FP64 router"}
        print(f"[bench] prefill {T}: {ms:.3f} ms/step, {out[str(T)]['tokens_per_s']:.0f} tokens/s, "
              f"{out[str(T)]['tflops']:.1f} TFLOP/s", file=sys.stderr, flush=True)
    return out


def main():
    a = parse()
    rank, world, local = dist_setup()
    if a.impl == "reference":
        impl_reference(a, rank, world)
        return
    import numpy as np
    import torch

    from coachwhip_b200 import _lib

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    pk = peaks()
    store, mods = build_stack(dev, a.layers)
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(dev)

    def maxall(v):
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    batches = [a.batch] if a.no_sweep else sorted({1, 4, 16, 64, a.batch})
    prefill_T = [] if a.no_prefill else (a.prefill_tokens or PREFILL_T)
    for m in mods:
        m.reserve(max(batches + prefill_T))  # one workspace for every captured graph
    sweep, graphs = {}, {}
    head = None
    ctx = _lib.ctx(local)
    for T in batches:
        x = synth_f32(T * H, stream(SEED, 0, T_IN), 1.0, dev).view(1, T, H)
        g, out = capture(mods, x, dev)
        graphs[T] = (g, x, out)
        barrier()
        if T == a.batch:
            with ClockSampler(local) as clk:
                ms = time_graph(g, a.steps, a.warmup, dev)
            clocks = clk.summary()
        else:
            ms = time_graph(g, max(5, a.steps // 2), a.warmup, dev)
        barrier()
        ms = maxall(ms)
        us = used_experts(mods, x)
        sweep[T] = {"tokens_per_s": world * T / (ms / 1e3), "ms_per_step": ms,
                    "unique_experts_mean": float(np.mean(us))}
        print(f"[bench] batch {T}: {ms:.3f} ms/step, {sweep[T]['tokens_per_s']:.1f} tokens/s, "
              f"{np.mean(us):.1f} experts/layer", file=sys.stderr, flush=True)
        if T == a.batch:
            head = (T, ms, clocks, us)

    T, ms, clocks, us = head
    g, x, _ = graphs[T]
    # kernels per step: counted by the library over one eager pass of the stack (a replay of the
    # graph issues the same kernels)
    l0 = _lib.lib().cwx_ctx_launches(ctx)
    run_stack(mods, x)
    torch.cuda.synchronize(dev)
    launches_per_step = _lib.lib().cwx_ctx_launches(ctx) - l0

    # per-phase CUDA-event durations: a second capture of the same stack with the library's phase
    # events inside the graph, replayed and read after each replay
    _lib.lib().cwx_ctx_reset_profile(ctx)
    _lib.lib().cwx_ctx_set_profiling(ctx, 1)
    gq = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        with torch.cuda.graph(gq, stream=s):
            run_stack(mods, x)
    torch.cuda.current_stream(dev).wait_stream(s)
    _lib.lib().cwx_ctx_set_profiling(ctx, 0)
    reps = 5
    tot = [0.0] * len(_lib.PHASES)
    for _ in range(reps):
        gq.replay()
        msv, _ = _lib.read_profile(local)
        tot = [p + q for p, q in zip(tot, msv)]
    _lib.lib().cwx_ctx_reset_profile(ctx)
    phase_ms = {n: tot[i] / reps for i, n in enumerate(_lib.PHASES)}
    del gq

    # algorithmic bytes of the expert-product launches over the stack
    g0, u0, d0 = store.banks[0]
    sh_gu = 2 * (I_S * H // 256 * 144)
    sh_d = H * I_S // 256 * 144
    act_gu = T * H * 4 + 2 * T * K * I * 4 + 2 * T * I_S * 4  # packed x read, gate/up rows written
    act_d = T * K * I * 4 + T * K * H * 4 + T * I_S * 4 + T * H * 4
    bytes_gu = sum(u * (g0.bytes_per_expert + u0.bytes_per_expert) + sh_gu + act_gu for u in us)
    bytes_d = sum(u * d0.bytes_per_expert + sh_d + act_d for u in us)
    gemv_ms = phase_ms["gate_up"] + phase_ms["down"]
    achieved = (bytes_gu + bytes_d) / (gemv_ms / 1e3) / 1e9
    expert_bytes = sum(u * (g0.bytes_per_expert + u0.bytes_per_expert + d0.bytes_per_expert) + sh_gu + sh_d for u in us)
    stack_frac = expert_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"]
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "k_gemv_traffic.json")))
        traffic = prof.get("dram_bytes_per_launch")
    except Exception:
        pass
    roofline = {"kernel": "k_gemv (gate/up + down expert products)", "bound": "hbm", "achieved": achieved,
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                "peak_source": "measured" if not pk.get("fallback") else "fallback",
                "launches_per_step": 2 * len(us), "algorithmic_bytes_per_step": bytes_gu + bytes_d,
                "kernel_ms_per_step": gemv_ms, "phase_ms_per_step": phase_ms,
                "stack_hbm_frac_expert_bytes": stack_frac}

    # end to end through the public API, host buffers, copies inside the timed region
    xh = x.detach().cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    st = torch.cuda.current_stream(dev)
    xd = torch.empty_like(x)
    e_steps = max(3, a.steps // 2)
    e0 = torch.cuda.Event(enable_timing=True)
    for i in range(a.warmup + e_steps):
        if i == a.warmup:
            barrier()
            e0.record(st)
        xd.copy_(xh, non_blocking=True)
        o = run_stack(mods, xd)
        oh.copy_(o, non_blocking=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e1.record(st)
    torch.cuda.synchronize(dev)
    e2e_ms = maxall(e0.elapsed_time(e1) / e_steps)
    _lib.status(local)

    # prefill runs the f32-activation policy (the reference GPU path's semantics, checked against
    # the O2 oracle): the same layers and banks, every product on the tensor cores
    from coachwhip_b200.moe import ExpertAct, StreamedMoe

    mods_f32 = [StreamedMoe(m.layer, m.gate, m.top_k, True, ExpertAct.Silu(), store, shared=m.shared,
                            act_mode=_lib.ACT_MODE_F32) for m in mods]
    for m in mods_f32:
        m.reserve(max(prefill_T) if prefill_T else 1)
    prefill = prefill_runs(mods_f32, prefill_T, a, dev, pk, maxall, barrier, world)
    del mods_f32
    ep = None
    if world > 1 and not a.no_ep:
        graphs.clear()  # the decode graphs are not replayed again; release before the EP banks
        ep = ep_runs(world, rank, local, a, maxall, barrier)
    c3 = None
    if not a.no_c3:
        graphs.clear()
        c3 = c3_runs(world, rank, local, a, pk, maxall, barrier)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        cpu = cpu_baseline(store, T)
    if rank == 0:
        line = {"metric": METRIC, "value": world * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "batch": T, "layers": a.layers, "parallelism": f"replicas x{world}",
                           "l2": "inputs larger than L2 (11.5 GB resident expert bank; ~10 GB read per step)",
                           "graph": "40-layer stack as one CUDA graph"},
                "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
                        "path": "StreamedMoe.forward x 40 via ctypes -> cwx_moe_forward"},
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks,
                "gpu_launches": int(launches_per_step * a.steps),
                "decode_sweep": {str(b): d for b, d in sweep.items()},
                "prefill": prefill, "expert_parallel": ep, "config3": c3}
        print(json.dumps(line), flush=True)
    graphs.clear()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
