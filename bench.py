"""Benchmark: coachwhip's MoE layer on B200 (headline = config 1).

Workload (`config.workload`): the Qwen3.6-35B-A3B-shaped decode stack, 40 MoE layers with every
expert resident in HBM: hidden 2048, 256 routed experts, top-8 renormalised, intermediate 512,
gate/up IQ2_S and down IQ3_S from N(0, 0.02) (seed 2), one Q4_K shared expert with a sigmoid
gate, router f32. One decode pass runs a batch of 64 tokens through the 40 layers
(x <- x + moe_l(x)); a step is DECODE_ITERS (16) decode passes of the batch, so 1,024 tokens per
step. Synthetic data: weights and inputs come from the library's seeded generator (no model
file); coachwhip_b200/workloads.py defines every configuration.

value:    tokens/s with inputs resident in HBM, each pass the 40-layer stack replayed as one
          CUDA graph (the expert banks, 11.5 GB, are far larger than L2: no flush needed).
e2e:      tokens/s through the public API (StreamedMoe.forward per layer, ctypes ->
          cwx_moe_forward) including, every pass, the pinned host->device copy of the batch and
          the device->host read of the result.
roofline: the expert-product kernel (k_gemv) at batch 64: algorithmic bytes (quantised weight
          bytes of the unique experts each launch reads + shared expert + activation traffic) over
          its CUDA-event duration (the library's phase events inside the graph), against the
          measured HBM copy bandwidth in MEASURED_PEAKS.json; `traffic` is the DRAM bytes of one
          captured launch (profiles/k_gemv_traffic.json, scaled per launch).
decode_sweep: batches 1, 4, 16, 64: tokens/s, unique experts per layer, expert-byte bandwidth and
          its fraction of the HBM peak, the k_gemv share and its own fraction.
prefill:  config 2 (the config-1 weights at 1500 and 4096 tokens, bf16 input widened to f32 at
          entry): one layer and the 40-layer stack; TFLOP/s against a dense FP8 GEMM peak measured
          here (torch._scaled_mm, e4m3) and the nominal 4.5 PFLOP/s, and against sustained bf16.
config3:  the gpt-oss-shaped stack (36 MXFP4 layers): decode 1 and 64 and prefill of 4096 tokens
          on one GPU; on N ranks the 4096-token prefill expert-parallel.
gdn_word: the linear-attention step before the MoE block (cwx_gdn_word: conv, norms, gates, delta
          rule, output norm and gate) over 30 layers of Qwen3-Next-shaped heads at 1 and 64
          sequences, HBM roofline on its algorithmic bytes; CPU baseline the oracle's restatement.
attn_word: the gated full-attention step (cwx_attn_word: q/k norms, rope, cache append, split-K
          softmax attention, gate) over 10 layers at 4096 cached rows, 1 and 64 sequences.
expert_parallel: config 4 (48 layers, 512 experts, Zipf-biased router, 8192 tokens): on one GPU
          the single-device layer (the anchor), on N ranks expert-parallel over NCCL with a per-phase
          breakdown and `ep_parity` (layer 0 on each rank's tokens against the single-device layer).
cpu_baseline: the vectorised CPU build of the same layer (oracle/fast.cpp: AVX2 integer dots for
          Q4_K x Q8_K as candle's x86 path, codebook-table dequantisation + f32 FMA dots for the IQ
          formats, which have no CPU path in the reference) on every host thread, one full layer of
          the same bank per call; cpu_baseline_scalar: the step-for-step restatement (oracle/).

usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cwx|reference] [--batch T]
                       [--no-sweep] [--no-prefill] [--no-ep] [--no-c3] [--no-gdn] [--no-cpu] [--c3-layers L]
                       [--prefill-tokens T ...] [--layers L]
For N > 1 it runs under torchrun: config 1 does not shard (each rank runs its own replica;
scaling "weak"); configs 3 and 4 shard their experts over the ranks (expert parallelism).
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

METRIC = "MoE-layer tokens/s (decode b=1-64, prefill 4K) and % of HBM/tensor roofline"
WORKLOAD = "config1 decode stack: 40 x MoE(H2048, E256, top8, I512, IQ2_S gate/up, IQ3_S down, Q4_K shared)"
DECODE_ITERS = 16  # decode passes of the batch per step
FP8_NOMINAL_TFLOPS = 4500.0  # B200 dense FP8, nominal
PREFILL_T = [1500, 4096]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="cwx", choices=["cwx", "reference"])
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--layers", type=int, default=40)
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-prefill", action="store_true")
    p.add_argument("--no-ep", action="store_true")
    p.add_argument("--no-c3", action="store_true", help="skip the config-3 (MXFP4, gpt-oss shape) runs")
    p.add_argument("--no-gdn", action="store_true",
                   help="skip the attention word steps before the MoE (linear and full attention)")
    p.add_argument("--gdn-seqs", type=int, nargs="*", default=[1, 64],
                   help="sequences per word step in the linear-attention runs (default 1 64)")
    p.add_argument("--c3-layers", type=int, default=36, help="config-3 layers (36; fewer for profiling)")
    p.add_argument("--c4-layers", type=int, default=48, help="config-4 layers (48; fewer for profiling)")
    p.add_argument("--prefill-tokens", type=int, nargs="*", default=None,
                   help="config-2 prefill sizes (default 1500 4096; one size for profiling)")
    return p.parse_args()


def config_dict(a, world):
    """The `config` of both arms' lines (identical, so the two lines name the same workload)."""
    return {"workload": WORKLOAD, "batch": a.batch, "layers": a.layers, "decode_iters_per_step": DECODE_ITERS,
            "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (11.5 GB resident expert bank; ~10 GB read per pass)",
            "graph": "40-layer stack as one CUDA graph, replayed once per decode pass"}


def dist_setup():
    import torch

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device(f"cuda:{local}"))
    return rank, world, local


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


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
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "fallback": True}


# ------------------------------------------------------------------------------------ helpers
def run_stack(mods, x):
    h = x
    for m in mods:
        h = m.forward(h, residual=h)
    return h


def capture(fn, dev):
    """fn() captured into a CUDA graph (run once outside capture first, to load the kernels)."""
    import torch

    fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            out = fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    return g, out


def time_graph(graph, steps, warmup, dev, reps=1):
    """ms per replay: `steps` timed steps of `reps` replays each, after `warmup` steps."""
    import torch

    for _ in range(warmup * reps):
        graph.replay()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps * reps):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / (steps * reps)


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


def phase_profile(mods, x, dev, local, reps=5):
    """Per-phase CUDA-event milliseconds of one pass of the stack: a capture with the library's
    phase events inside the graph, replayed and read after each replay."""
    import torch

    from coachwhip_b200 import _lib

    ctx = _lib.ctx(local)
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
    tot = [0.0] * len(_lib.PHASES)
    for _ in range(reps):
        gq.replay()
        msv, _ = _lib.read_profile(local)
        tot = [p + q for p, q in zip(tot, msv)]
    _lib.lib().cwx_ctx_reset_profile(ctx)
    del gq
    return {n: tot[i] / reps for i, n in enumerate(_lib.PHASES)}


def gemv_bytes(cfg, us, T):
    """Algorithmic bytes of the two expert-product launches of each layer at batch T: the unique
    experts' quantised bytes, the shared expert, the packed activation rows read and the product
    rows written."""
    H, I, Is, K = cfg.hidden, cfg.inter, cfg.shared_inter, cfg.top_k
    from coachwhip_b200.moe import row_bytes

    e_gu = row_bytes(cfg.gate_type, H) * I + row_bytes(cfg.up_type, H) * I
    e_d = row_bytes(cfg.down_type, I) * H
    sh_gu = 2 * row_bytes(cfg.sh_type, H) * Is
    sh_d = row_bytes(cfg.sh_type, Is) * H
    act_gu = T * H * 4 + 2 * T * K * I * 4 + 2 * T * Is * 4
    act_d = T * K * I * 4 + T * K * H * 4 + T * Is * 4 + T * H * 4
    gu = sum(u * e_gu + sh_gu + act_gu for u in us)
    d = sum(u * e_d + sh_d + act_d for u in us)
    expert = sum(u * (e_gu + e_d) + sh_gu + sh_d for u in us)
    return gu + d, expert


def fused_bytes(cfg, us, T):
    """Algorithmic bytes of the fused decode layer per pass: the router weights, the unique
    experts' and the shared expert's quantised bytes, the input, residual and output rows."""
    _, expert = gemv_bytes(cfg, us, T)
    return expert + len(us) * (cfg.n_experts * cfg.hidden * 4 + 3 * T * cfg.hidden * 4)


# ------------------------------------------------------------------------------ CPU baselines
def cpu_layer(store_banks, shared, router_w):
    """Layer 0 of config 1 for the CPU builds (bank bytes downloaded from the GPU)."""
    import oracle as O

    from coachwhip_b200 import workloads as W

    cfg = W.CONFIGS["C1"]
    g, u, d = store_banks
    L = dict(hidden=cfg.hidden, n_experts=cfg.n_experts, top_k=cfg.top_k, inter=cfg.inter, norm_topk_prob=1,
             gate_type=cfg.gate_type, up_type=cfg.up_type, down_type=cfg.down_type, act=O.ACT_SILU,
             gate_bank=g.download(), up_bank=u.download(), down_bank=d.download(),
             router_w=router_w.cpu().numpy(), shared_inter=cfg.shared_inter, sh_gate_type=cfg.sh_type,
             sh_up_type=cfg.sh_type, sh_down_type=cfg.sh_type, sh_gate=shared.gate.download(),
             sh_up=shared.up.download(), sh_down=shared.down.download(),
             sh_gate_inp=shared.gate_inp.cpu().numpy())
    return L


def cpu_layer_host():
    """Layer 0 of config 1 synthesised on the host (the reference arm has no GPU)."""
    import oracle as O

    from coachwhip_b200 import workloads as W

    cfg = W.CONFIGS["C1"]
    st = lambda t: W.stream(cfg.seed, 0, t)  # noqa: E731
    E, H, I, Is = cfg.n_experts, cfg.hidden, cfg.inter, cfg.shared_inter
    return dict(hidden=H, n_experts=E, top_k=cfg.top_k, inter=I, norm_topk_prob=1, gate_type=cfg.gate_type,
                up_type=cfg.up_type, down_type=cfg.down_type, act=O.ACT_SILU,
                gate_bank=O.synth_matrix(cfg.gate_type, st(W.T_GATE), 0, E, I, H, 0.02),
                up_bank=O.synth_matrix(cfg.up_type, st(W.T_UP), 0, E, I, H, 0.02),
                down_bank=O.synth_matrix(cfg.down_type, st(W.T_DOWN), 0, E, H, I, 0.02),
                router_w=O.normal(st(W.T_RW), 0, E * H, 0.02).reshape(E, H), shared_inter=Is,
                sh_gate_type=cfg.sh_type, sh_up_type=cfg.sh_type, sh_down_type=cfg.sh_type,
                sh_gate=O.synth_matrix(cfg.sh_type, st(W.T_SG), 0, 1, Is, H, 0.02),
                sh_up=O.synth_matrix(cfg.sh_type, st(W.T_SU), 0, 1, Is, H, 0.02),
                sh_down=O.synth_matrix(cfg.sh_type, st(W.T_SD), 0, 1, H, Is, 0.02),
                sh_gate_inp=O.normal(st(W.T_SGI), 0, H, 0.02))


def cpu_input(T):
    import oracle as O

    from coachwhip_b200 import workloads as W

    cfg = W.CONFIGS["C1"]
    return O.normal(W.stream(cfg.input_seed, 0, W.T_IN), 0, T * cfg.hidden, 1.0).reshape(T, cfg.hidden)


def time_cpu(fn, budget_s, max_calls):
    fn()  # warm (tables, page cache)
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= max_calls:
            return el / n, n


def cpu_baselines(L, T, layers):
    """Both CPU builds of one full layer at batch T on every host thread."""
    import oracle as O

    th = host_threads()
    O.set_threads(th)
    x = cpu_input(T)
    out = {}
    for kind, fn, budget, label in (
            ("fast", lambda: O.moe_forward_fast(L, x), 8.0,
             "the vectorised CPU build (oracle/fast.cpp: AVX2/FMA; Q4_K x Q8_K integer dots as candle's x86 path, "
             "codebook-table dequantisation and f32 dots for IQ2_S/IQ3_S, which have no CPU path in the reference)"),
            ("scalar", lambda: O.moe_forward(L, x, O.MODE_CANDLE), 6.0,
             "the step-for-step C++ restatement of the reference's CPU arithmetic (oracle/, vec_dot_unopt order)")):
        per_layer, n = time_cpu(fn, budget, 50)
        out[kind] = {"value": T / (per_layer * layers), "unit": "tokens/s", "cores": th, "kind": "port",
                     "cpu": cpu_model(),
                     "sample": f"{n} calls of one full config-1 layer (256 experts, batch {T}) through {label}; "
                               f"tokens/s = batch / ({layers} x per-layer time)",
                     "per_layer_ms": per_layer * 1e3}
    return out


def impl_reference(a, rank, world):
    """The reference arm: the CPU port of the reference's layer on the host cores (rank 0)."""
    if rank != 0:
        return
    import oracle as O

    th = host_threads()
    O.set_threads(th)  # every host thread, whatever OMP_NUM_THREADS the launcher set
    T = a.batch
    L = cpu_layer_host()
    x = cpu_input(T)
    for _ in range(max(1, a.warmup)):
        O.moe_forward_fast(L, x)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        O.moe_forward_fast(L, x)  # one layer per step: a bounded sample of the stack
    per_layer = (time.perf_counter() - t0) / a.steps
    v = T / (per_layer * a.layers)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": per_layer * 1e3, "layers_timed_per_step": 1,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(a, world),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": th, "kind": "port", "cpu": cpu_model(),
                             "sample": f"each step: one full config-1 layer (256 experts, one pass of a {T}-token "
                                       f"batch) through the vectorised CPU build of the reference's layer "
                                       f"(oracle/fast.cpp, AVX2/FMA; the reference has no CPU path for IQ2_S/IQ3_S, "
                                       f"whose shader math it restates); ms_per_step is that one layer; tokens/s = "
                                       f"batch / ({a.layers} x per-layer time)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU parts
def fp8_peak(dev):
    """Dense FP8 (e4m3) GEMM throughput of a plain library call (torch._scaled_mm), 8192^3."""
    import torch

    try:
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        f = lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)  # noqa: E731
        for _ in range(3):
            f()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = 0.0
        for _ in range(5):
            e0.record()
            for _ in range(5):
                f()
            e1.record()
            torch.cuda.synchronize(dev)
            best = max(best, 5 * 2 * n ** 3 / (e0.elapsed_time(e1) / 1e3) / 1e12)
        del a, b
        return {"tflops": best, "how": "torch._scaled_mm e4m3 x e4m3 -> bf16, 8192^3, best of 5 x 5 (burst)"}
    except Exception as e:  # the roofline then uses the nominal figure only
        return {"tflops": None, "how": f"unavailable: {type(e).__name__}: {e}"[:200]}


GDN_SHAPE = dict(n_k=16, n_v=32, dk=128, dv=128, taps=4, cycle=1)  # Qwen3-Next / Qwen3.6 linear attention
GDN_LAYERS = 30  # the linear-attention layers of a 40-layer stack (every fourth layer is full attention)


def gdn_bytes(n_seq, n_k, n_v, dk, dv, taps, **_):
    """Algorithmic bytes of one word step over n_seq sequences: each head's memory read and
    written, the conv window read and written, qkv, z, beta/alpha in, o out; the layer's conv
    weights, dt_bias, a and norm_w once per launch."""
    ch = 2 * n_k * dk + n_v * dv
    per_seq = 4 * (2 * n_v * dk * dv + 2 * (taps - 1) * ch + ch + n_v * dv + 2 * n_v + n_v * dv)
    return n_seq * per_seq + 4 * (ch * taps + 2 * n_v + dv)


def gdn_runs(world, rank, local, a, pk, maxall, barrier):
    """The Gated DeltaNet word step before the MoE block (cwx_gdn_word): GDN_LAYERS layers, each
    with its own constants, memory and conv window, one word of n_seq sequences per layer, the
    layers replayed as one CUDA graph; memory updated in place. Also the oracle's restatement of the
    reference kernel on one host thread (one layer, one sequence), the CPU baseline of this step."""
    import ctypes

    import numpy as np
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200 import workloads as W
    from coachwhip_b200.gdn import GdnWord

    dev = torch.device(f"cuda:{local}")
    sh = GDN_SHAPE
    n_k, n_v, dk, dv, taps = sh["n_k"], sh["n_v"], sh["dk"], sh["dv"], sh["taps"]
    ch = 2 * n_k * dk + n_v * dv
    out = {"config": f"{GDN_LAYERS} x GatedDeltaNet word step (n_k {n_k}, n_v {n_v}, dk {dk}, dv {dv}, {taps} taps, "
                     "key heads cycled), f32; synthetic constants and inputs from the seeded generator",
           "layers": GDN_LAYERS,
           "kernel": "k_gdn_head (one CTA per head and sequence; other head shapes take k_gdn_word)"}
    rng_key = lambda l, t: W.stream(7, l, t)  # noqa: E731
    consts = []
    for l in range(GDN_LAYERS):
        consts.append(dict(conv_w=W.normal(ch * taps, rng_key(l, 0), 0.4, local).view(ch, taps),
                           dt_bias=W.normal(n_v, rng_key(l, 1), 1.0, local),
                           a=-torch.exp(W.normal(n_v, rng_key(l, 2), 1.0, local).abs()),
                           norm_w=1.0 + W.normal(dv, rng_key(l, 3), 0.1, local)))
    for n_seq in a.gdn_seqs:
        ops, words = [], []
        for l, c in enumerate(consts):
            s = W.normal(n_seq * n_v * dk * dv, rng_key(l, 10 + n_seq), 0.1, local).view(n_seq, n_v, dk, dv)
            cs = W.normal(n_seq * (taps - 1) * ch, rng_key(l, 11 + n_seq), 1.0, local).view(n_seq, taps - 1, ch)
            ops.append(GdnWord(cs, c["conv_w"], c["dt_bias"], c["a"], c["norm_w"], s, n_k, n_v, dk, dv, taps, True,
                               1e-6))
            words.append(dict(qkv=W.normal(n_seq * ch, rng_key(l, 12 + n_seq), 1.0, local).view(n_seq, ch),
                              z=W.normal(n_seq * n_v * dv, rng_key(l, 13 + n_seq), 1.0, local).view(n_seq, -1),
                              ba=W.normal(n_seq * 2 * n_v, rng_key(l, 14 + n_seq), 1.0, local).view(n_seq, -1),
                              o=torch.empty(n_seq, n_v * dv, device=dev),
                              cv=torch.empty_like(cs)))
        layers_c = [op.layer() for op in ops]

        def step():
            # the launches go to the stream being captured; the window moves to a buffer of its own
            # (conv_out may not alias conv_state)
            st = torch.cuda.current_stream(dev)
            for op, w, L in zip(ops, words, layers_c):
                _lib.check(_lib.lib().cwx_gdn_word(ctypes.byref(L), n_seq, w["qkv"].data_ptr(), w["z"].data_ptr(),
                                                   w["ba"].data_ptr(), op.conv_state.data_ptr(), op.s.data_ptr(),
                                                   w["o"].data_ptr(), op.s.data_ptr(), w["cv"].data_ptr(),
                                                   st.cuda_stream))

        g, _ = capture(step, dev)
        barrier()
        ms = maxall(time_graph(g, max(10, a.steps), a.warmup, dev))
        del g
        _lib.status(local)
        alg = GDN_LAYERS * gdn_bytes(n_seq, **sh)
        achieved = alg / (ms / 1e3) / 1e9
        out[f"n_seq_{n_seq}"] = {"ms_per_stack": ms, "us_per_layer": ms * 1e3 / GDN_LAYERS,
                                 "tokens_per_s": world * n_seq / (ms / 1e3),
                                 "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                                              "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                                              "algorithmic_bytes_per_launch": alg / GDN_LAYERS,
                                              "peak_source": "measured" if not pk.get("fallback") else "fallback"},
                                 "l2": "each layer its own memory (2.1 MB per sequence, "
                                       f"{GDN_LAYERS * n_seq * 2.1e-3:.2f} GB over the stack), read and written "
                                       "once per word"}
        print(f"[bench] gdn word, {n_seq} sequences: {ms * 1e3 / GDN_LAYERS:.2f} us/layer, "
              f"{achieved:.0f} GB/s ({achieved / pk['hbm_gbs']:.3f} of HBM)", file=sys.stderr, flush=True)
        del ops, words
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not a.no_cpu:
        import oracle as O

        rng = np.random.default_rng(0)
        f = np.float32
        args = [rng.standard_normal(ch).astype(f), rng.standard_normal(n_v * dv).astype(f),
                rng.standard_normal(2 * n_v).astype(f), rng.standard_normal((taps - 1, ch)).astype(f),
                (0.4 * rng.standard_normal((ch, taps))).astype(f), rng.standard_normal(n_v).astype(f),
                -np.exp(np.abs(rng.standard_normal(n_v))).astype(f), (1 + 0.1 * rng.standard_normal(dv)).astype(f),
                (0.1 * rng.standard_normal((n_v, dk, dv))).astype(f)]
        O.gdn_word(n_k, n_v, dk, dv, taps, True, 1e-6, *args)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 3.0:
            O.gdn_word(n_k, n_v, dk, dv, taps, True, 1e-6, *args)
            n += 1
        per = (time.perf_counter() - t0) / n
        out["cpu_baseline"] = {"value": 1.0 / (GDN_LAYERS * per), "unit": "tokens/s (one sequence)", "cores": 1,
                               "kind": "port", "per_layer_ms": per * 1e3,
                               "sample": f"{n} calls of one layer's word step for one sequence through the oracle's "
                                         "restatement of the reference kernel (oracle/gdn.cpp, one thread); "
                                         f"tokens/s = 1 / ({GDN_LAYERS} x per-layer time)"}
    return out


ATTN_SHAPE = dict(n_head=16, n_kv=2, hd=256, rot=64)  # Qwen3-Next / Qwen3.6 gated full attention
ATTN_LAYERS = 10  # the full-attention layers of a 40-layer stack
ATTN_CTX = 4096   # cached rows per sequence when the timed word arrives


def attn_bytes(n_seq, ctx, n_head, n_kv, hd, **_):
    """Algorithmic bytes of one full-attention word over n_seq sequences with ctx cached rows:
    the K and V rows read (ctx + 1 each, the new row included), the new row written, qg, k, v in
    and the output out."""
    return n_seq * 4 * (2 * n_kv * (ctx + 1) * hd + 2 * n_kv * hd + 2 * n_head * hd + 2 * n_kv * hd + n_head * hd)


def attn_runs(world, rank, local, a, pk, maxall, barrier):
    """The gated full-attention word step (cwx_attn_word) at ATTN_CTX cached rows: ATTN_LAYERS layers,
    each its own cache, one word of n_seq sequences per layer, replayed as one CUDA graph (the
    cache lengths stay put: each replay writes the same row)."""
    import ctypes

    import numpy as np
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200 import workloads as W
    from coachwhip_b200.attn import FullAttn, KvCache

    dev = torch.device(f"cuda:{local}")
    sh = ATTN_SHAPE
    n_head, n_kv, hd, rot = sh["n_head"], sh["n_kv"], sh["hd"], sh["rot"]
    cap = ATTN_CTX + 64
    out = {"config": f"{ATTN_LAYERS} x gated full-attention word step (n_head {n_head}, n_kv {n_kv}, hd {hd}, "
                     f"rope on {rot}), {ATTN_CTX} cached rows per sequence, f32 caches; synthetic inputs",
           "layers": ATTN_LAYERS,
           "kernel": "k_attn_part (32 cache rows of one kv head per CTA, bulk copies) between k_attn_prep and "
                     "k_attn_combine"}
    key = lambda l, t: W.stream(8, l, t)  # noqa: E731
    for n_seq in a.gdn_seqs:
        layers = []
        for l in range(ATTN_LAYERS):
            att = FullAttn(1.0 + W.normal(hd, key(l, 0), 0.1, local), 1.0 + W.normal(hd, key(l, 1), 0.1, local),
                           n_head, n_kv, hd, rot, 1e7, 1e-6)
            cache = KvCache(n_seq, n_kv, cap, hd, dev)
            cache.k.copy_(W.normal(cache.k.numel(), key(l, 2), 0.5, local).view_as(cache.k))
            cache.v.copy_(W.normal(cache.v.numel(), key(l, 3), 1.0, local).view_as(cache.v))
            cache.len.fill_(ATTN_CTX)
            layers.append(dict(att=att, L=att.layer(), cache=cache,
                               qg=W.normal(n_seq * n_head * 2 * hd, key(l, 4), 1.0, local),
                               kn=W.normal(n_seq * n_kv * hd, key(l, 5), 1.0, local),
                               vn=W.normal(n_seq * n_kv * hd, key(l, 6), 1.0, local),
                               o=torch.empty(n_seq, n_head * hd, device=dev)))
        ctx = _lib.ctx(local)

        def step():
            st = torch.cuda.current_stream(dev)  # (the stream being captured)
            for y in layers:
                c = y["cache"]
                _lib.check(_lib.lib().cwx_attn_word(ctx, ctypes.byref(y["L"]), n_seq, c.cap, y["qg"].data_ptr(),
                                                    y["kn"].data_ptr(), y["vn"].data_ptr(), c.k.data_ptr(),
                                                    c.v.data_ptr(), c.len.data_ptr(), c.len.data_ptr(),
                                                    y["o"].data_ptr(), st.cuda_stream))

        g, _ = capture(step, dev)
        barrier()
        ms = maxall(time_graph(g, max(10, a.steps), a.warmup, dev))
        del g
        _lib.status(local)
        alg = ATTN_LAYERS * attn_bytes(n_seq, ATTN_CTX, **sh)
        achieved = alg / (ms / 1e3) / 1e9
        out[f"n_seq_{n_seq}"] = {"ms_per_stack": ms, "us_per_layer": ms * 1e3 / ATTN_LAYERS,
                                 "tokens_per_s": world * n_seq / (ms / 1e3),
                                 "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                                              "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                                              "algorithmic_bytes_per_launch": alg / ATTN_LAYERS,
                                              "peak_source": "measured" if not pk.get("fallback") else "fallback"},
                                 "l2": f"each layer its own cache ({2 * n_kv * cap * hd * 4 * n_seq / 1e6:.0f} MB), "
                                       f"{ATTN_LAYERS} layers per replay"}
        print(f"[bench] attn word, {n_seq} sequences, {ATTN_CTX} rows: {ms * 1e3 / ATTN_LAYERS:.2f} us/layer, "
              f"{achieved:.0f} GB/s ({achieved / pk['hbm_gbs']:.3f} of HBM)", file=sys.stderr, flush=True)
        del layers
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not a.no_cpu:
        import oracle as O

        rng = np.random.default_rng(0)
        f = np.float32
        cap_c = ATTN_CTX + 1
        args = [rng.standard_normal((n_head, 2 * hd)).astype(f), rng.standard_normal((n_kv, hd)).astype(f),
                rng.standard_normal((n_kv, hd)).astype(f), np.ones(hd, f), np.ones(hd, f),
                rng.standard_normal((n_kv, cap_c, hd)).astype(f), rng.standard_normal((n_kv, cap_c, hd)).astype(f)]
        O.attn_word(n_head, n_kv, hd, rot, 1e-6, 1e7, ATTN_CTX, ATTN_CTX, *args)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 3.0:
            O.attn_word(n_head, n_kv, hd, rot, 1e-6, 1e7, ATTN_CTX, ATTN_CTX, *args)
            n += 1
        per = (time.perf_counter() - t0) / n
        out["cpu_baseline"] = {"value": 1.0 / (ATTN_LAYERS * per), "unit": "tokens/s (one sequence)", "cores": 1,
                               "kind": "port", "per_layer_ms": per * 1e3,
                               "sample": f"{n} calls of one layer's word step for one sequence at {ATTN_CTX} rows "
                                         "through the oracle's restatement (oracle/gdn.cpp cwo_attn_word, one "
                                         f"thread); tokens/s = 1 / ({ATTN_LAYERS} x per-layer time)"}
    return out


def prefill_runs(cfg, mods, Ts, a, dev, local, pk, fp8, maxall, barrier, world):
    """Config 2: one layer and the 40-layer stack at 1500 and 4096 tokens, bf16 input widened to
    f32 at entry (the reference casts to f32 at the layer's entry), f32 activation policy."""
    import torch

    from coachwhip_b200 import workloads as W

    out = {}
    tpk = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    for T in Ts:
        xb = W.make_input(cfg, T, local).to(torch.bfloat16).view(1, T, cfg.hidden)
        res = {}
        for nl in (1, len(mods)):
            ms_ = mods[:nl]
            g, _ = capture(lambda: run_stack(ms_, xb.to(torch.float32)), dev)
            barrier()
            ms = maxall(time_graph(g, max(3, a.steps // 4), max(2, a.warmup // 2), dev))
            del g
            fl = nl * cfg.flops(T)
            tf = fl / (ms / 1e3) / 1e12
            r = {"layers": nl, "ms_per_step": ms, "tokens_per_s": world * T / (ms / 1e3), "tflops": tf,
                 "frac_fp8_nominal": tf / FP8_NOMINAL_TFLOPS, "frac_bf16_sustained_measured": tf / tpk}
            if fp8.get("tflops"):
                r["frac_fp8_measured"] = tf / fp8["tflops"]
            res["1_layer" if nl == 1 else f"{nl}_layers"] = r
            print(f"[bench] prefill {T} x {nl} layers: {ms:.3f} ms, {tf:.1f} TFLOP/s", file=sys.stderr, flush=True)
        out[str(T)] = res
    return out


def c3_runs(world, rank, local, a, pk, maxall, barrier, fp8=None):
    """Config 3: decode batches 1 and 64 and prefill of 4096 tokens on one GPU (36-layer stack as
    CUDA graphs); on N ranks the 4096-token prefill expert-parallel (128 / N experts per rank)."""
    import numpy as np
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200 import workloads as W
    from coachwhip_b200.moe import ExpertStore

    cfg = W.CONFIGS["C3"]
    dev = torch.device(f"cuda:{local}")
    desc = ("config 3: 36 x MoE(H2880, E128, top4, I2880, MXFP4 gate/up/down with per-expert biases, clamped "
            "SwiGLU 1.702/7.0, router bias, no shared expert); candle activation policy (Q8_0 codes)")
    nl = a.c3_layers
    t0 = time.time()
    epr = cfg.n_experts // world
    b_exp = cfg.expert_bytes() + (2 * cfg.inter + cfg.hidden) * 4
    res = {"config": desc, "layers": nl}
    if world > 1:
        from coachwhip_b200.ep import CudaEngine, EpComm, LibraryExpertParallelMoe

        T = 4096
        per = T // world
        comm = EpComm(local, world, rank)
        mods = []
        for l in range(nl):
            lay = W.build_layer(cfg, l, local, first=rank * epr, n_local=epr)
            eng = CudaEngine(lay.router_w, cfg.top_k, True, lay.act, lay.banks, world, rank, gate_bias=lay.router_b)
            eng._keep = lay
            mods.append(LibraryExpertParallelMoe(eng, comm, per))
        torch.cuda.synchronize(dev)
        res["bank_synthesis_s"] = time.time() - t0
        x = W.make_input(cfg, T, local)[rank * per:(rank + 1) * per].contiguous().view(1, per, cfg.hidden)
        for _ in range(max(1, a.warmup // 2)):
            run_stack(mods, x)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 2
        e0.record()
        for _ in range(reps):
            run_stack(mods, x)
        e1.record()
        torch.cuda.synchronize(dev)
        ms = maxall(e0.elapsed_time(e1) / reps)
        _lib.status(local)
        fl = nl * cfg.flops(T)
        res["prefill"] = {"tokens": T, "tokens_per_rank": per, "ranks": world, "experts_per_rank": epr,
                          "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "tflops": fl / (ms / 1e3) / 1e12,
                          "transport": "cwx_ep_forward: NCCL inside libcwx, fixed-capacity exchanges, no host sync",
                          "timing": f"CUDA events over {reps} eager passes, max over ranks"}
        # decode batches 1 and 64 spread over the ranks (a rank may hold no token: it still takes
        # part in both exchanges and runs the picks the others send it)
        res["decode"] = {}
        for Td in (1, 64):
            lo, hi = Td * rank // world, Td * (rank + 1) // world
            capd = max(1, (Td + world - 1) // world)
            for m in mods:
                m.cap_tokens = capd
            xd = W.make_input(cfg, Td, local)[lo:hi].contiguous().view(1, hi - lo, cfg.hidden)
            for _ in range(3):
                run_stack(mods, xd)
            barrier()
            e0.record()
            for _ in range(5):
                run_stack(mods, xd)
            e1.record()
            torch.cuda.synchronize(dev)
            msd = maxall(e0.elapsed_time(e1) / 5)
            res["decode"][str(Td)] = {"ms_per_step": msd, "tokens_per_s": Td / (msd / 1e3),
                                      "timing": "CUDA events over 5 eager passes, max over ranks"}
        _lib.status(local)
        del mods
        comm.close()
        return res
    store = ExpertStore([])
    layers = [W.build_layer(cfg, l, local, store=store) for l in range(nl)]
    mods = [lay.moe for lay in layers]
    torch.cuda.synchronize(dev)
    res["bank_synthesis_s"] = time.time() - t0
    res["bank_gb"] = nl * cfg.n_experts * b_exp / 1e9
    for m in mods:
        m.reserve(4096)
    res["decode"] = {}
    for T in (1, 64):
        x = W.make_input(cfg, T, local).view(1, T, cfg.hidden)
        g, _ = capture(lambda: run_stack(mods, x), dev)
        ms = time_graph(g, max(5, a.steps // 2), a.warmup, dev)
        del g
        us = used_experts(mods, x)
        eb = sum(us) * b_exp + nl * cfg.n_experts * cfg.hidden * 4  # experts read + router weights
        ph = phase_profile(mods, x, dev, local)
        res["decode"][str(T)] = {"tokens_per_s": T / (ms / 1e3), "ms_per_step": ms,
                                 "unique_experts_mean": float(np.mean(us)),
                                 "hbm_gbs_expert_bytes": eb / (ms / 1e3) / 1e9,
                                 "hbm_frac": eb / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
                                 "phase_ms_per_step": {k: v for k, v in ph.items() if v > 0}}
        print(f"[bench] config 3 decode {T}: {ms:.3f} ms/step, {T / (ms / 1e3):.1f} tokens/s", file=sys.stderr,
              flush=True)
    T = 4096
    x = W.make_input(cfg, T, local).view(1, T, cfg.hidden)
    g, _ = capture(lambda: run_stack(mods, x), dev)
    ms = time_graph(g, 3, max(1, a.warmup // 2), dev)
    del g
    fl = nl * cfg.flops(T)
    res["prefill"] = {"tokens": T, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
                      "tflops": fl / (ms / 1e3) / 1e12, "frac_fp8_nominal": fl / (ms / 1e3) / 1e12 / FP8_NOMINAL_TFLOPS,
                      "path": ("tcgen05 grouped products (k_mma<MXFP4>: weights decoded to f16 A tiles, exact for "
                               "banks whose block scales lie in [104, 140]; activations as f16 hi + lo under the "
                               "Q8_0 policy; clamped-SwiGLU and bias epilogues)")}
    if fp8 and fp8.get("tflops"):
        res["prefill"]["frac_fp8_measured"] = res["prefill"]["tflops"] / fp8["tflops"]
    print(f"[bench] config 3 prefill {T}: {ms:.3f} ms/step", file=sys.stderr, flush=True)
    _lib.status(local)
    return res


def ep_runs(world, rank, local, a, maxall, barrier):
    """Config 4 expert-parallel: 48 layers, 8192 tokens split over the ranks, f32 policy."""
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200 import workloads as W
    from coachwhip_b200.ep import CudaEngine
    from coachwhip_b200.moe import ExpertStore

    cfg = W.CONFIGS["C4"]
    dev = torch.device(f"cuda:{local}")
    nl = a.c4_layers
    T = 8192
    per = T // world
    desc = ("config 4: 48 x MoE(H2048, E512, top10, I512, IQ3_S gate/up, Q4_K down, Q4_K shared, Zipf(1.1) router "
            "bias); f32 activation policy")
    fl = nl * cfg.flops(T)
    if world == 1:  # the anchor: the single-device layer on the whole batch
        store = ExpertStore([])
        mods = [W.build_layer(cfg, l, local, act_mode=_lib.ACT_MODE_F32, store=store).moe for l in range(nl)]
        for m in mods:
            m.reserve(T)
        x = W.make_input(cfg, T, local).view(1, T, cfg.hidden)
        g, _ = capture(lambda: run_stack(mods, x), dev)
        ms = time_graph(g, 3, 2, dev)
        del g
        _lib.status(local)
        return {"config": desc, "layers": nl, "tokens": T, "ranks": 1, "experts_per_rank": cfg.n_experts,
                "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "tflops": fl / (ms / 1e3) / 1e12,
                "path": "single-device cwx_moe_forward (no exchange), CUDA graph of the 48 layers"}
    import numpy as np
    import torch.distributed as dist

    from coachwhip_b200.ep import EpComm, LibraryExpertParallelMoe, balanced_placement, expert_lists

    epr = cfg.n_experts // world
    comm = EpComm(local, world, rank)
    layers = []
    # Expert placement per layer from a calibration batch (2048 tokens of another input stream):
    # its picks per expert, spread over the ranks by balanced_placement (rank 0 decides, the
    # others receive it). The Zipf bias sends two thirds of the picks to ten experts, so the
    # contiguous ranges would leave one rank with about twice the mean load.
    n_cal = 2048
    xc = W.normal(n_cal * cfg.hidden, W.stream(cfg.input_seed + 101, 0, W.T_IN), 1.0, local).view(n_cal, cfg.hidden)
    loads = {"contiguous": [], "balanced": []}
    for l in range(nl):
        rw, rb = W.router(cfg, l, local)
        lg = xc @ rw.t() + (rb if rb is not None else 0)
        cnt = torch.bincount(lg.topk(cfg.top_k, dim=1).indices.reshape(-1), minlength=cfg.n_experts).cpu().numpy()
        del rw, rb, lg
        slot = torch.from_numpy(balanced_placement(cnt, world)).to(dev)
        dist.broadcast(slot, 0)
        slot = slot.cpu().numpy()
        per_rank = np.zeros(world)
        np.add.at(per_rank, slot // epr, cnt)
        loads["balanced"].append(float(per_rank.max() / per_rank.mean()))
        loads["contiguous"].append(float(cnt.reshape(world, epr).sum(1).max() / per_rank.mean()))
        lay = W.build_layer(cfg, l, local, act_mode=_lib.ACT_MODE_F32, experts=expert_lists(slot, world)[rank])
        eng = CudaEngine(lay.router_w, cfg.top_k, True, lay.act, lay.banks, world, rank, gate_bias=lay.router_b,
                         shared=lay.shared, act_mode=_lib.ACT_MODE_F32, placement=slot)
        eng._keep = lay
        layers.append(LibraryExpertParallelMoe(eng, comm, per))
    x = W.make_input(cfg, T, local)[rank * per:(rank + 1) * per].contiguous().view(1, per, cfg.hidden)
    for _ in range(max(1, a.warmup // 2)):
        run_stack(layers, x)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        run_stack(layers, x)
    e1.record()
    torch.cuda.synchronize(dev)
    ms = maxall(e0.elapsed_time(e1) / reps)
    # per-phase breakdown of one more pass: the library's phase events (max over ranks)
    ctx = _lib.ctx(local)
    _lib.lib().cwx_ctx_reset_profile(ctx)
    _lib.lib().cwx_ctx_set_profiling(ctx, 1)
    barrier()
    run_stack(layers, x)
    _lib.lib().cwx_ctx_set_profiling(ctx, 0)
    msv, _ = _lib.read_profile(local)
    _lib.lib().cwx_ctx_reset_profile(ctx)
    ph = {n: maxall(msv[i]) for i, n in enumerate(_lib.PHASES) if n.startswith("ep_")}
    # parity: layer 0 on this rank's tokens against the single-device layer (all 512 experts)
    taps = {}
    out_ep = layers[0].forward(x, taps=taps)[0]
    full = W.build_layer(cfg, 0, local, act_mode=_lib.ACT_MODE_F32)
    ftaps = {}
    out_1 = full.moe.forward(x, taps=ftaps)[0]
    _lib.status(local)
    rel = float((out_ep - out_1).double().norm() / out_1.double().norm())
    ids_eq = bool(torch.equal(taps["ids"].view(-1), ftaps["ids"].view(-1)))
    rel = maxall(rel)
    ids_all = maxall(0.0 if ids_eq else 1.0) == 0.0
    del full, layers
    comm.close()
    return {"config": desc, "layers": nl, "tokens": T, "tokens_per_rank": per, "ranks": world,
            "experts_per_rank": epr, "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3),
            "tflops": fl / (ms / 1e3) / 1e12, "phase_ms_per_step": ph,
            "ep_parity": {"rel_l2": rel, "ids_equal": ids_all, "bar": 1e-3,
                          "what": "layer 0 on each rank's tokens vs the single-device layer; max over ranks"},
            "transport": "cwx_ep_forward: NCCL inside libcwx, fixed-capacity exchanges (counts read on the "
                         "device), no host synchronisation in a layer",
            "placement": {"how": "balanced_placement of a 2048-token calibration batch's picks per expert, per "
                                 "layer (equal experts per rank)",
                          "max_over_mean_rank_picks": {k: float(np.mean(v)) for k, v in loads.items()}},
            "timing": f"CUDA events over {reps} eager passes of the {nl} layers, max over ranks"}


# ------------------------------------------------------------------------------------- main
def main():
    a = parse()
    rank, world, local = dist_setup()
    if a.impl == "reference":
        impl_reference(a, rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    import numpy as np
    import torch

    from coachwhip_b200 import _lib
    from coachwhip_b200 import workloads as W
    from coachwhip_b200.moe import ExpertStore

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    pk = peaks()
    cfg = W.CONFIGS["C1"]
    store = ExpertStore([])
    layers = [W.build_layer(cfg, l, local, store=store) for l in range(a.layers)]
    mods = [lay.moe for lay in layers]
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
    sweep, head = {}, None
    ctx = _lib.ctx(local)
    for T in batches:
        x = W.make_input(cfg, T, local).view(1, T, cfg.hidden)
        g, _ = capture(lambda: run_stack(mods, x), dev)
        barrier()
        if T == a.batch:
            with ClockSampler(local) as clk:
                ms = time_graph(g, a.steps, a.warmup, dev, reps=DECODE_ITERS)
            clocks = clk.summary()
        else:
            ms = time_graph(g, max(5, a.steps // 2), a.warmup, dev)
        del g
        barrier()
        ms = maxall(ms)
        us = used_experts(mods, x)
        ph = phase_profile(mods, x, dev, local)
        alg, expert = gemv_bytes(cfg, us, T)
        gemv_ms = ph["gate_up"] + ph["down"]
        sweep[T] = {"tokens_per_s": world * T / (ms / 1e3), "ms_per_pass": ms,
                    "unique_experts_mean": float(np.mean(us)),
                    "hbm_gbs_expert_bytes": expert / (ms / 1e3) / 1e9,
                    "hbm_frac_expert_bytes": expert / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
                    "phase_ms_per_pass": ph}
        if gemv_ms > 0:  # the grouped products (the fused decode layer has no separate product launches)
            sweep[T].update({"k_gemv_ms_per_pass": gemv_ms, "k_gemv_share": gemv_ms / ms,
                             "k_gemv_hbm_frac": alg / (gemv_ms / 1e3) / 1e9 / pk["hbm_gbs"]})
        if ph.get("decode_fused", 0) > 0:
            fb = fused_bytes(cfg, us, T)
            sweep[T].update({"path": "fused decode layer (k_decode_layer, one cooperative launch per layer)",
                             "k_decode_layer_ms_per_pass": ph["decode_fused"],
                             "k_decode_layer_hbm_frac": fb / (ph["decode_fused"] / 1e3) / 1e9 / pk["hbm_gbs"]})
        print(f"[bench] batch {T}: {ms:.3f} ms/pass, {sweep[T]['tokens_per_s']:.1f} tokens/s, "
              f"{np.mean(us):.1f} experts/layer, expert bytes {sweep[T]['hbm_frac_expert_bytes']:.3f} of HBM",
              file=sys.stderr, flush=True)
        if T == a.batch:
            head = (T, ms, clocks, us, ph, alg)

    T, ms, clocks, us, phase_ms, alg = head
    x = W.make_input(cfg, T, local).view(1, T, cfg.hidden)
    # kernels per pass: counted by the library over one eager pass (a replay issues the same kernels)
    l0 = _lib.lib().cwx_ctx_launches(ctx)
    run_stack(mods, x)
    torch.cuda.synchronize(dev)
    launches_per_pass = _lib.lib().cwx_ctx_launches(ctx) - l0

    gemv_ms = phase_ms["gate_up"] + phase_ms["down"]
    if gemv_ms > 0:
        achieved = alg / (gemv_ms / 1e3) / 1e9
        traffic, traffic_src = None, None
        try:
            prof = json.load(open(os.path.join(ROOT, "profiles", "k_gemv_traffic.json")))
            traffic, traffic_src = prof.get("dram_bytes_per_launch"), prof.get("source")
        except Exception:
            pass
        roofline = {"kernel": "k_gemv (gate/up + down expert products)", "bound": "hbm", "achieved": achieved,
                    "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                    "traffic_source": traffic_src,
                    "peak_source": "measured" if not pk.get("fallback") else "fallback",
                    "launches_per_pass": 2 * len(us), "algorithmic_bytes_per_launch": alg / (2 * len(us)),
                    "algorithmic_bytes_per_pass": alg, "kernel_ms_per_pass": gemv_ms,
                    "stack_hbm_frac_expert_bytes": sweep[T]["hbm_frac_expert_bytes"]}
    else:  # the fused decode layer: one launch per layer does all of it
        fb = fused_bytes(cfg, us, T)
        fms = phase_ms["decode_fused"]
        roofline = {"kernel": "k_decode_layer (the whole layer, one launch)", "bound": "hbm",
                    "achieved": fb / (fms / 1e3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                    "frac": fb / (fms / 1e3) / 1e9 / pk["hbm_gbs"],
                    "traffic": 13.0e6, "traffic_source": "ncu --set full capture of profiles/k_decode_layer_c1_b1.md "
                                                         "(one layer at b = 1, dram bytes read + written)",
                    "peak_source": "measured" if not pk.get("fallback") else "fallback",
                    "launches_per_pass": len(us), "algorithmic_bytes_per_launch": fb / len(us),
                    "algorithmic_bytes_per_pass": fb, "kernel_ms_per_pass": fms,
                    "stack_hbm_frac_expert_bytes": sweep[T]["hbm_frac_expert_bytes"]}

    # end to end through the public API, host buffers, copies inside the timed region
    xh = x.detach().cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    st = torch.cuda.current_stream(dev)
    xd = torch.empty_like(x)
    e_steps = max(3, a.steps // 4)
    e0 = torch.cuda.Event(enable_timing=True)
    for i in range(a.warmup + e_steps):
        if i == a.warmup:
            barrier()
            e0.record(st)
        for _ in range(DECODE_ITERS):
            xd.copy_(xh, non_blocking=True)
            o = run_stack(mods, xd)
            oh.copy_(o, non_blocking=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e1.record(st)
    torch.cuda.synchronize(dev)
    e2e_ms = maxall(e0.elapsed_time(e1) / (e_steps * DECODE_ITERS))
    _lib.status(local)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        lay0 = layers[0]
        cpu = cpu_baselines(cpu_layer(lay0.banks, lay0.shared, lay0.router_w), T, a.layers)

    # prefill (config 2): the same layers and banks under the f32 policy (the reference GPU
    # path's semantics, checked against the O2 oracle); routed and shared products on the tensor cores
    from coachwhip_b200.moe import StreamedMoe

    fp8 = fp8_peak(dev) if (prefill_T or not a.no_c3) else None
    prefill = None
    if prefill_T:
        mods_f32 = [StreamedMoe(m.layer, m.gate, m.top_k, True, m.act, store, shared=m.shared,
                                act_mode=_lib.ACT_MODE_F32) for m in mods]
        for m in mods_f32:
            m.reserve(max(prefill_T))
        prefill = prefill_runs(cfg, mods_f32, prefill_T, a, dev, local, pk, fp8, maxall, barrier, world)
        prefill["fp8_peak"] = fp8
        del mods_f32
    del mods, layers, store
    torch.cuda.empty_cache()
    gdn = None if a.no_gdn else gdn_runs(world, rank, local, a, pk, maxall, barrier)
    attn = None if a.no_gdn else attn_runs(world, rank, local, a, pk, maxall, barrier)
    c3 = None
    if not a.no_c3:
        c3 = c3_runs(world, rank, local, a, pk, maxall, barrier, fp8)
        torch.cuda.empty_cache()
    ep = None
    if not a.no_ep:
        ep = ep_runs(world, rank, local, a, maxall, barrier)

    if rank == 0:
        steps_tokens = world * T * DECODE_ITERS
        line = {"metric": METRIC, "value": world * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms * DECODE_ITERS, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config_dict(a, world), "tokens_per_step": steps_tokens,
                "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": DECODE_ITERS * T * cfg.hidden * 4,
                        "d2h_bytes_per_step": DECODE_ITERS * T * cfg.hidden * 4,
                        "path": "StreamedMoe.forward x 40 via ctypes -> cwx_moe_forward, per decode pass"},
                "roofline": roofline, "phase_ms_per_pass": phase_ms,
                "cpu_baseline": cpu["fast"] if cpu else None,
                "cpu_baseline_scalar": cpu["scalar"] if cpu else None, "clocks": clocks,
                "gpu_launches": int(launches_per_pass * DECODE_ITERS * a.steps),
                "decode_sweep": {str(b): d for b, d in sweep.items()},
                "prefill": prefill, "expert_parallel": ep, "config3": c3, "gdn_word": gdn,
                "attn_word": attn}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
