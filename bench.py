"""Benchmark of the INT4 MLP/MoE prefill path on B200 (driver contract: one JSON line).

Headline workload ("C2"): the dense INT4 SwiGLU MLP block, 4096
tokens, hidden 4096, intermediate 12288 -- prepare(x) -> gate|up GEMM -> fused SwiGLU
packing -> down GEMM, one clefq_mlp C-ABI call per step.  Synthetic data (seed 0 + rank):
activations BF16 N(0,1), weight codes uniform in [-8, 7] (uniform random tiled words),
one f32 scale per output row |N(0, 0.02)|/7.  The L2 (126 MB) is flushed by a 256 MB
write between timed steps; each step is timed with CUDA events on the launching stream.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl clefq|reference]

Multi-GPU: one process per GPU (torchrun); every rank runs its own 4096-token block with
replicated weights (data-parallel replicas, no collective on the data path): weak scaling.
The `secondary` line runs the C4 MoE layer expert-parallel (clefq_moe_ep_layer, dispatch and
return stored into peers' buffers by the kernels; the NCCL all-to-all composition timed
beside it) and the `tensor_parallel` line one C2 block split over the ranks (clefq_tp_mlp).
`e2e` streams host rows through clefq.mlp_host, copies included.  Further lines: `c1` (BASELINE
configs[0], one 128 x 2048 -> 768 projection, GPU and CPU), `c3` (configs[2], the 28-layer INT4
decoder prefill at 2048 tokens, attention glue timed apart) and `c5` (configs[4], 48 MoE layers
at 8192 tokens per GPU, expert-parallel when N > 1).
--impl reference: the reference's CPU semantics (the C/OpenMP oracle port; the reference
itself is Rust + hrx-rs on an AMD gfx1151 and cannot run here) on the host cores, rank 0.
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

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
sys.path.insert(0, ROOT)

METRIC = "INT4 MLP/MoE prefill tokens/s"
M, HIDDEN, INTER = 4096, 4096, 12288          # C2
MOE_T, MOE_H, MOE_I, MOE_E, MOE_K = 8192, 2048, 768, 128, 8   # C4
C1_M, C1_K, C1_N = 128, 2048, 768                               # C1
C3_S, C3_H, C3_I, C3_L, C3_QH, C3_KVH, C3_HD = 2048, 2560, 9728, 28, 32, 8, 128   # C3
C5_L = 48                                                       # C5: 48 x the C4 MoE layer
FLUSH_BYTES = 256 << 20


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p.get("hbm_gbs", 6650.0), p.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None, "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def all_min(world, flag: bool) -> bool:
    """True only if every rank's flag is true."""
    if world == 1:
        return bool(flag)
    import torch.distributed as dist
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def all_max(world, value: float) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------------
# synthetic weights (BASELINE: codes uniform in [-8, 7], scales |N(0, 0.02)|/7)
# ---------------------------------------------------------------------------------------
def rand_weight_dev(clefq, rows, cols, gen):
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows * cols // 8,), dtype=torch.int32, device="cuda", generator=gen)
    scales = (torch.randn(rows, device="cuda", generator=gen).abs() * 0.02 / 7).float()
    return clefq.QuantizedWeight(codes, scales, rows, cols, clefq.stride_for(cols), 4)


def rand_weight_host(rng, rows, cols):
    codes = rng.integers(0, 2 ** 32, size=rows * cols // 8, dtype=np.uint64).astype(np.uint32)
    scales = (np.abs(rng.standard_normal(rows)) * 0.02 / 7).astype(np.float32)
    return codes, scales, rows


# GPU spin (~0.2 ms) queued after each step's L2 flush and before its start event: the host
# has enqueued the whole step by the time the start event executes, so a step's time is its
# device time and not the host's launch path (which the e2e line measures, host buffers
# included).
LEAD = 400_000


def time_steps(fn, steps, flush, lead_cycles=0):
    """Device time of each step (CUDA events on the launching stream), L2 flushed before
    every step; returns per-step milliseconds.  lead_cycles > 0 queues a GPU spin after
    the flush so the host has enqueued the step before its start event executes: a
    kernel shorter than the host's launch path is then timed, not the host."""
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        flush.fill_(1)
        if lead_cycles:
            torch.cuda._sleep(lead_cycles)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


# ---------------------------------------------------------------------------------------
# CPU legs (oracle port): only here, the tests and smoke() may run oracle/
# ---------------------------------------------------------------------------------------
def cpu_mlp_sample(tokens: int, min_seconds: float, threads: int):
    from oracle import oracle as o
    rng = np.random.default_rng(0)
    g, u, d = rand_weight_host(rng, INTER, HIDDEN), rand_weight_host(rng, INTER, HIDDEN), rand_weight_host(rng, HIDDEN, INTER)
    x = o.f32_to_bf16(rng.standard_normal((tokens, HIDDEN)).astype(np.float32))
    reps, t0 = 0, time.perf_counter()
    while True:
        o.mlp_block(x, g, u, d, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds and reps >= 2:
            break
    return tokens * reps / el, reps, el


def run_config(world):
    """The workload both arms report (the reference arm times bounded samples of it)."""
    return {"workload": "C2 dense INT4 SwiGLU MLP block", "tokens_per_gpu": M, "hidden": HIDDEN,
            "intermediate": INTER, "parallelism": f"dp{world} (replicas)" if world > 1 else "single GPU",
            "l2": "flushed (256 MB write) before every timed step"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    from oracle import oracle as o
    rng = np.random.default_rng(0)
    g, u, d = rand_weight_host(rng, INTER, HIDDEN), rand_weight_host(rng, INTER, HIDDEN), rand_weight_host(rng, HIDDEN, INTER)
    sample = 256
    x = o.f32_to_bf16(rng.standard_normal((sample, HIDDEN)).astype(np.float32))
    for _ in range(args.warmup):
        o.mlp_block(x, g, u, d, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        o.mlp_block(x, g, u, d, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1000 * sum(times) / len(times)
    value = sample / (ms / 1000)
    desc = (f"{sample} of the 4096 C2 tokens per step through the full-size weights "
            f"(hidden {HIDDEN}, intermediate {INTER}), oracle port of the reference semantics on "
            f"{threads} host threads (OpenMP)")
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 codes, int32 dot, f32 epilogue", "data": "synthetic (seed 0)",
            "impl": "reference",
            "config": run_config(world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_c1(clefq, gen, flush, args, world, rank, i8_peak):
    """project_quantized of 128 BF16 rows (K = 2048) through a 768-row
    int4 weight -- packing of the rows plus the GEMM, timed per call with the L2 flushed in
    between; F32 output as the config states.  Rank 0 at N = 1 also times the CPU oracle on
    the same call."""
    m, k, n = C1_M, C1_K, C1_N
    w = rand_weight_dev(clefq, n, k, gen)
    x = torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
    step = lambda: clefq.project_quantized(x, w, out_dtype=torch.float32)   # noqa: E731
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    times = time_steps(step, max(20, min(args.steps, 200)), flush, lead_cycles=LEAD)
    ms = all_max(world, statistics.median(times))
    ops = 2.0 * m * n * k
    out = {"workload": "C1 single INT4 GEMM: 128 x 2048 BF16 rows packed, then 768 x 2048 int4 weight, F32 out",
           "calls": len(times), "ms_per_call": ms, "tokens_per_s": world * m / (ms / 1000),
           "tops": ops / (ms / 1000) / 1e12, "frac_of_int8_peak": ops / (ms / 1000) / 1e12 / i8_peak,
           "gpu_launches_per_call": 2,
           "note": "latency-bound: 3 pair tiles on 148 SMs; the median of the per-call device times"}
    if rank == 0 and world == 1 and not args.skip_cpu:
        from oracle import oracle as o
        threads = len(os.sched_getaffinity(0))
        rng = np.random.default_rng(0)
        wt, ws, _ = rand_weight_host(rng, n, k)
        xh = o.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
        reps, t0 = 0, time.perf_counter()
        while True:
            _, codes, scales, _ = o.prepare(xh, 4, o.stride_for(k), threads=threads)
            o.gemm(codes, scales, wt, ws, n, k, out_f32=True, threads=threads)
            reps += 1
            el = time.perf_counter() - t0
            if el >= 3.0 and reps >= 5:
                break
        out["cpu_baseline"] = {"value": m * reps / el, "unit": "tokens/s", "cores": threads, "kind": "port",
                               "ms_per_call": 1000 * el / reps,
                               "sample": f"{reps} whole C1 calls ({el:.1f} s), CPU oracle port"}
    return out


def run_c3(clefq, gen, flush, args, world, rank, i8_peak):
    """a 28-layer decoder prefill, 2048 tokens, hidden 2560, 32 query / 8
    KV heads of 128, MLP 9728, every projection INT4.  Per layer (the reference's backbone
    call sites, src/backbone.rs:866-907): RMSNorm fused into the packing of the residual
    stream -> one q|k|v projection (the three weights stacked by rows) -> causal GQA SDPA
    (BF16, torch: attention is not on the INT4 path) -> o projection with the residual fused
    -> normalized_mlp (RMSNorm packing, gate|up, SwiGLU packing, down + residual).  Rotary
    embeddings are left out (glue outside the INT4 path).  Every rank runs its own sequence
    (replicas).  The int4 time is the step minus the attention glue, both CUDA-event timed."""
    import torch.nn.functional as F
    S, H, I, L = C3_S, C3_H, C3_I, C3_L
    qd, kvd = C3_QH * C3_HD, C3_KVH * C3_HD
    layers = []
    for _ in range(L):
        layers.append((rand_weight_dev(clefq, qd + 2 * kvd, H, gen), rand_weight_dev(clefq, H, qd, gen),
                       rand_weight_dev(clefq, I, H, gen), rand_weight_dev(clefq, I, H, gen),
                       rand_weight_dev(clefq, H, I, gen),
                       (torch.randn(H, device="cuda", generator=gen) * 0.02).to(torch.bfloat16),
                       (torch.randn(H, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)))
    x0 = torch.randn(S, H, device="cuda", generator=gen).to(torch.bfloat16)
    ws = torch.empty(clefq.lib().clefq_mlp_workspace_size(S, H, I), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    att_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]

    def step(record=False):
        h = x0
        for li, (wqkv, wo, g, u, d, n1, n2) in enumerate(layers):
            a = clefq.prepare(h, 4, clefq.stride_for(H), clefq.PREP_NORM, n1)
            qkv = clefq.project_prepared(S, wqkv, a)
            if record:
                att_ev[li][0].record(stream)
            q = qkv[:, :qd].view(S, C3_QH, C3_HD).transpose(0, 1).unsqueeze(0)
            k = qkv[:, qd:qd + kvd].view(S, C3_KVH, C3_HD).transpose(0, 1).unsqueeze(0)
            v = qkv[:, qd + kvd:].view(S, C3_KVH, C3_HD).transpose(0, 1).unsqueeze(0)
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            attn = o[0].transpose(0, 1).reshape(S, qd)
            if record:
                att_ev[li][1].record(stream)
            h = clefq.project_quantized(attn, wo, residual=h)
            h = clefq.normalized_mlp(h, n2, g, u, d, workspace=ws)
        return h

    for _ in range(max(2, args.warmup)):
        step()
    torch.cuda.synchronize()
    clefq.status()
    barrier(world)
    totals, atts = [], []
    for _ in range(max(3, min(args.steps, 10))):
        flush.fill_(1)
        torch.cuda._sleep(LEAD)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        step(record=True)
        t1.record(stream)
        torch.cuda.synchronize()
        totals.append(t0.elapsed_time(t1))
        atts.append(sum(a.elapsed_time(b) for a, b in att_ev))
    clefq.status()
    ms = all_max(world, statistics.median(totals))
    att_ms = all_max(world, statistics.median(atts))
    int4_ms = ms - att_ms
    ops = L * 2.0 * S * (H * (qd + 2 * kvd) + qd * H + 3 * H * I)
    out = {"workload": "C3 INT4 decoder prefill: 28 layers, 2048 tokens, hidden 2560, GQA 32q/8kv x 128, MLP 9728; "
                       "q|k|v, o, gate, up, down all INT4 (RMSNorm fused into packing; SDPA glue in BF16)",
           "tokens_per_s": world * S / (ms / 1000), "ms_per_step": ms, "attention_glue_ms": att_ms,
           "int4_ms": int4_ms, "int4_tokens_per_s": world * S / (int4_ms / 1000),
           "int_ops_per_step": ops, "frac_of_int8_peak_int4_part": ops / (int4_ms / 1000) / 1e12 / i8_peak,
           "gpu_launches_per_layer": 8, "parallelism": f"dp{world} (replicas)" if world > 1 else "single GPU",
           "note": "rotary embeddings left out; the attention glue (torch SDPA, causal, GQA) is timed with CUDA events "
                   "and reported apart"}
    if rank == 0 and world == 1 and not args.skip_cpu:
        from oracle import oracle as o
        threads = len(os.sched_getaffinity(0))
        rng = np.random.default_rng(3)
        tok = 128
        wqkv, wo = rand_weight_host(rng, qd + 2 * kvd, H), rand_weight_host(rng, H, qd)
        g, u, d = rand_weight_host(rng, I, H), rand_weight_host(rng, I, H), rand_weight_host(rng, H, I)
        n1 = o.f32_to_bf16((rng.standard_normal(H) * 0.02).astype(np.float32))
        xh = o.f32_to_bf16(rng.standard_normal((tok, H)).astype(np.float32))
        attn_h = o.f32_to_bf16(rng.standard_normal((tok, qd)).astype(np.float32))
        reps, t0 = 0, time.perf_counter()
        while True:
            _, c, sc, _ = o.prepare(xh, 4, o.stride_for(H), o.NORM, n1, threads=threads)
            o.gemm(c, sc, *wqkv, H, threads=threads)
            _, c, sc, _ = o.prepare(attn_h, 4, o.stride_for(qd), threads=threads)
            r = o.gemm(c, sc, *wo, qd, residual=xh, threads=threads)
            o.normalized_mlp_block(r, n1, g, u, d, threads=threads)
            reps += 1
            el = time.perf_counter() - t0
            if el >= 5.0 and reps >= 2:
                break
        per_layer_s = el / reps * (S / tok)
        out["cpu_baseline"] = {"value": S / (per_layer_s * L), "unit": "tokens/s", "cores": threads, "kind": "port",
                               "sample": f"{reps} x one layer's INT4 projections on {tok} tokens ({el:.1f} s), "
                                         f"scaled x{S // tok} tokens and x{L} layers; attention not included"}
    del layers
    return out


def run_c5(clefq, gen, flush, args, world, rank, i8_peak):
    """full-depth MoE prefill -- 48 layers of the C4 MoE layer, each with
    its own router and expert weights, 8192 tokens per GPU (65,536 at 8 GPUs, 16 experts per
    GPU), run back to back with the residual added after every layer.  N > 1: every layer is one clefq_moe_ep_layer call
    (experts sharded over the ranks).  The router linear runs fused with the router inside each
    layer.  The interleaved attention core is not on the INT4 path and is not timed here."""
    per = MOE_E // world
    layers = []
    for _ in range(C5_L):
        wr = torch.randn(MOE_E, MOE_H, device="cuda", generator=gen).to(torch.bfloat16)
        gate = rand_weight_dev(clefq, per * MOE_I, MOE_H, gen)
        up = rand_weight_dev(clefq, per * MOE_I, MOE_H, gen)
        down = rand_weight_dev(clefq, per * MOE_H, MOE_I, gen)
        layers.append((wr, gate, up, down))
    x0 = torch.randn(MOE_T, MOE_H, device="cuda", generator=gen).to(torch.bfloat16)
    comm = None
    if world > 1:
        from clefq.comm import Comm
        from clefq.ep import ExpertShard, ep_layer_region_bytes, omni_moe_ep_fused
        cap = world * MOE_T * MOE_K
        comm = Comm(ep_layer_region_bytes(MOE_T, MOE_H, MOE_K, world, cap))
        ws = torch.empty(clefq.lib().clefq_moe_ep_layer_workspace_size(MOE_T, MOE_H, MOE_I, MOE_E, MOE_K, world, cap),
                         dtype=torch.uint8, device="cuda")
        shards = [ExpertShard(g, u, d, rank * per, per, MOE_E, MOE_I) for _, g, u, d in layers]
    else:
        ws = torch.empty(clefq.lib().clefq_moe_workspace_size(MOE_T, MOE_H, MOE_I, MOE_E, MOE_K), dtype=torch.uint8,
                         device="cuda")
    out_buf = torch.empty((MOE_T, MOE_H), dtype=torch.bfloat16, device="cuda")

    def step():
        h = x0
        for li, (wr, g, u, d) in enumerate(layers):
            if world > 1:
                omni_moe_ep_fused(h, None, shards[li], comm, MOE_K, recv_cap=cap, workspace=ws, out=out_buf,
                                  router_weight=wr)
            else:
                clefq.omni_moe(h, None, g, u, d, workspace=ws, router_weight=wr, out=out_buf)
            h = h + out_buf
        return h

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    clefq.status()
    barrier(world)
    times = time_steps(step, max(3, min(args.steps, 5)), flush, lead_cycles=LEAD)
    clefq.status()
    ms = all_max(world, statistics.median(times))
    if comm is not None:
        comm.close()
    ops = C5_L * 2.0 * MOE_T * MOE_K * (MOE_H * 2 * MOE_I + MOE_I * MOE_H)
    out = {"workload": f"C5 full-depth MoE prefill: 48 x the C4 MoE layer (own weights per layer), {MOE_T} tokens "
                       f"per GPU ({world * MOE_T} in all), {per} experts per GPU, residual after each layer",
           "tokens_per_s": world * MOE_T / (ms / 1000), "ms_per_step": ms, "ms_per_layer": ms / C5_L,
           "int_ops_per_rank_per_step": ops, "frac_of_int8_peak": ops / (ms / 1000) / 1e12 / i8_peak,
           "parallelism": f"ep{world}: one clefq_moe_ep_layer call per layer" if world > 1 else "single GPU",
           "note": "router linear fused with the router and residual add inside the step; the interleaved "
                   "attention core is not on the INT4 path and not timed"}
    if rank == 0 and world == 1 and not args.skip_cpu:
        from oracle import oracle as o
        threads = len(os.sched_getaffinity(0))
        rng = np.random.default_rng(5)
        tok = 512
        g, u, d = (rand_weight_host(rng, MOE_E * MOE_I, MOE_H), rand_weight_host(rng, MOE_E * MOE_I, MOE_H),
                   rand_weight_host(rng, MOE_E * MOE_H, MOE_I))
        xh = o.f32_to_bf16(rng.standard_normal((tok, MOE_H)).astype(np.float32))
        lg = o.f32_to_bf16((rng.standard_normal((tok, MOE_E)) * 40).astype(np.float32))
        reps, t0 = 0, time.perf_counter()
        while True:
            o.moe_layer(xh, lg, (g[0], g[1], MOE_I), (u[0], u[1], MOE_I), (d[0], d[1], MOE_H), threads=threads)
            reps += 1
            el = time.perf_counter() - t0
            if el >= 5.0 and reps >= 2:
                break
        per_layer_s = el / reps * (MOE_T / tok)
        out["cpu_baseline"] = {"value": MOE_T / (per_layer_s * C5_L), "unit": "tokens/s", "cores": threads,
                               "kind": "port", "sample": f"{reps} x one C4 MoE layer on {tok} tokens ({el:.1f} s), "
                                                         f"scaled x{MOE_T // tok} tokens and x{C5_L} layers"}
    del layers
    return out


# ---------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------
def run_clefq(args, world, rank, local):
    import clefq
    clefq.lib()
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    i8_peak = 2 * bf16_peak   # B200: dense int8 tensor rate is twice dense bf16
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + rank)
    gate, up, down = (rand_weight_dev(clefq, INTER, HIDDEN, gen), rand_weight_dev(clefq, INTER, HIDDEN, gen),
                      rand_weight_dev(clefq, HIDDEN, INTER, gen))
    x = torch.randn(M, HIDDEN, device="cuda", generator=gen).to(torch.bfloat16)
    ws = torch.empty(clefq.lib().clefq_mlp_workspace_size(M, HIDDEN, INTER), dtype=torch.uint8, device="cuda")
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    step = lambda: clefq.mlp(x, gate, up, down, workspace=ws)   # noqa: E731

    sampler = ClockSampler(local)
    sampler.start()
    # W warm-up steps at least; keep warming for ~1 s so the clock samples see the load.
    t0, done = time.perf_counter(), 0
    while done < args.warmup or time.perf_counter() - t0 < 1.0:
        step()
        done += 1
        if done % 50 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    clefq.status()
    barrier(world)
    torch.cuda.synchronize()
    times = time_steps(step, args.steps, flush, lead_cycles=LEAD)
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop()
    clefq.status()
    ms_local = sum(times) / len(times)
    ms = all_max(world, ms_local)
    value = world * M / (ms / 1000)

    # ---- per-kernel timing of the same step, each launch as clefq_mlp issues it -------
    # The dominant kernel is the gate|up GEMM: one launch over both weight matrices
    # (N = 2 x 12288, K = 4096) with SwiGLU in its epilogue (clefq_gemm_swiglu_s8), writing
    # the BF16 hidden rows; then the plain packing of those rows and the down GEMM
    # (N = 4096, K = 12288).
    a = clefq.prepare(x, 4, clefq.stride_for(HIDDEN))
    gu = torch.zeros((M, INTER), dtype=torch.bfloat16, device="cuda")
    ktimes = {}
    reps = max(5, min(args.steps, 50))

    def gemm_gu():
        clefq.project_swiglu_prepared(M, gate, up, a, out=gu)
    gemm_gu()
    hid = clefq.prepare(gu, 4, clefq.stride_for(INTER))
    out = torch.empty((M, HIDDEN), dtype=torch.bfloat16, device="cuda")

    def gemm_down():
        clefq._call("clefq_gemm_s8", clefq._stream(), 4, clefq._ptr(hid.operand), INTER, clefq._ptr(hid.scales), M,
                    clefq._ptr(down.codes), clefq._ptr(down.scales), HIDDEN, INTER, None, 0, 0, clefq._ptr(out),
                    HIDDEN)
    lead = LEAD
    for name, fn in (("gemm_gate_up", gemm_gu), ("gemm_down", gemm_down)):
        fn()
        ktimes[name] = statistics.median(time_steps(fn, reps, flush, lead))
    ktimes["prepare_x"] = statistics.median(time_steps(lambda: clefq.prepare(x, 4, clefq.stride_for(HIDDEN)), reps,
                                                       flush, lead))
    ktimes["prepare_hidden"] = statistics.median(time_steps(
        lambda: clefq.prepare(gu, 4, clefq.stride_for(INTER)), reps, flush, lead))
    # Rooflines of the two GEMM launches exactly as clefq_mlp issues them; algorithmic work
    # 2*M*N*K each (gate|up: N = 2 x INTER, K = HIDDEN; down: N = HIDDEN, K = INTER).
    traffic_tab = load_traffic()
    gu_ops = 2.0 * M * (2 * INTER) * HIDDEN
    gu_achieved = gu_ops / (ktimes["gemm_gate_up"] / 1000) / 1e12
    down_ops = 2.0 * M * HIDDEN * INTER
    down_achieved = down_ops / (ktimes["gemm_down"] / 1000) / 1e12

    # ---- end to end through the public API with host buffers ---------------------------
    # clefq.mlp_host (clefq_mlp_host): pinned host rows in, pinned host rows out, K calls back
    # to back as a server would issue them.  Every step copies its 4096 input rows to the GPU
    # and its output rows back inside the timed region; the L2 is flushed on the compute
    # stream before each step.  Within a call the rows go through in chunks; with
    # streaming=True the next call's input copies overlap this call's kernels.  The first call
    # waits for the start event; the region ends when the last output copy is done.  Chunk
    # sizes are tried on this box and the fastest is reported.  The stream runs at least 100
    # calls, so the pipeline's fill (the first input copy) and drain (the last call's kernels
    # and output copy, ~1.3 ms together) are spread as a serving loop spreads them.
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((M, HIDDEN), dtype=torch.bfloat16).pin_memory()
    e2e_steps = args.e2e_steps if args.e2e_steps > 0 else max(100, min(args.steps, 200))
    stream = torch.cuda.current_stream()
    best = None
    for chunk in (1024, 2048, 4096):
        hws = torch.empty(clefq.lib().clefq_mlp_host_workspace_size(chunk, HIDDEN, INTER, 0), dtype=torch.uint8,
                          device="cuda")
        done = torch.cuda.Event()

        def e2e_run(k):
            for i in range(k):
                flush.fill_(1)
                clefq.mlp_host(x_host, gate, up, down, out=out_host, chunk_rows=chunk, workspace=hws, sync=False,
                               streaming=i > 0, done_event=done)
            stream.wait_event(done)
        e2e_run(3)
        torch.cuda.synchronize()
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        e2e_run(e2e_steps)
        t1.record(stream)
        torch.cuda.synchronize()
        t_ms = all_max(world, t0.elapsed_time(t1) / e2e_steps)
        if best is None or t_ms < best[0]:
            best = (t_ms, chunk)
        del hws
    e2e_ms, e2e_chunk = best

    # ---- secondary workload: the C4 MoE layer (8192 tokens, 128 experts, top-8) --------
    moe = None
    if not args.skip_moe:
        mx = torch.randn(MOE_T, MOE_H, device="cuda", generator=gen).to(torch.bfloat16)
        wr = torch.randn(MOE_E, MOE_H, device="cuda", generator=gen).to(torch.bfloat16)
        # the NCCL composition routes from precomputed logits; the fused layers take the
        # router weight and run the router linear fused with the router inside the layer
        logits = mx @ wr.t()
        # The expert weights are the same on every rank (one seed): rank r keeps its slice, and
        # the full set gives the single-GPU result each rank's expert-parallel output must equal.
        wgen = torch.Generator(device="cuda")
        wgen.manual_seed(2000)
        mg = rand_weight_dev(clefq, MOE_E * MOE_I, MOE_H, wgen)
        mu = rand_weight_dev(clefq, MOE_E * MOE_I, MOE_H, wgen)
        md = rand_weight_dev(clefq, MOE_E * MOE_H, MOE_I, wgen)
        mws = torch.empty(clefq.lib().clefq_moe_workspace_size(MOE_T, MOE_H, MOE_I, MOE_E, MOE_K),
                          dtype=torch.uint8, device="cuda")
        nccl_ms = None
        parity = None
        parity_paths = None
        if world > 1:
            # expert parallel: this rank owns MOE_E / world experts and its own MOE_T tokens;
            # one clefq_moe_ep_layer call per step (records and products stored into the peers'
            # symmetric buffers by the kernels), the NCCL all-to-all composition timed beside it
            from clefq.comm import Comm
            from clefq.ep import ep_layer_region_bytes, omni_moe_ep, omni_moe_ep_fused, shard_experts
            shard = shard_experts(mg, mu, md, MOE_E, MOE_I, MOE_H, rank, world)
            cap = world * MOE_T * MOE_K
            ecomm = Comm(ep_layer_region_bytes(MOE_T, MOE_H, MOE_K, world, cap))
            ews = torch.empty(clefq.lib().clefq_moe_ep_layer_workspace_size(MOE_T, MOE_H, MOE_I, MOE_E, MOE_K, world,
                                                                            cap), dtype=torch.uint8, device="cuda")
            eout = torch.empty((MOE_T, MOE_H), dtype=torch.bfloat16, device="cuda")
            nstep = lambda: omni_moe_ep(mx, logits, shard, MOE_K)   # noqa: E731
            # parity before timing: both expert-parallel paths against clefq_moe on one GPU
            ref = clefq.omni_moe(mx, logits, mg, mu, md, workspace=mws)
            nccl_out = nstep()[0]
            # the fused layer from the precomputed logits, then with the router linear fused in
            lout, _ = omni_moe_ep_fused(mx, logits, shard, ecomm, MOE_K, recv_cap=cap, workspace=ews)
            _, eroutes = omni_moe_ep_fused(mx, None, shard, ecomm, MOE_K, recv_cap=cap, workspace=ews, out=eout,
                                           router_weight=wr)
            rroutes = torch.empty((MOE_T, 2 * MOE_K), dtype=torch.float32, device="cuda")
            ref_fused = clefq.omni_moe(mx, None, mg, mu, md, workspace=mws, router_weight=wr, routes_out=rroutes)
            torch.cuda.synchronize()
            clefq.status()
            same_fused = torch.equal(eout.view(torch.int16), ref_fused.view(torch.int16))
            same_nccl = torch.equal(nccl_out.view(torch.int16), ref.view(torch.int16))
            parity = all_min(world, same_fused and same_nccl)
            parity_paths = {"fused": all_min(world, same_fused), "nccl": all_min(world, same_nccl),
                            "fused_routes": all_min(world, torch.equal(eroutes, rroutes)),
                            "fused_from_logits": all_min(world, torch.equal(lout.view(torch.int16),
                                                                            ref.view(torch.int16)))}
            del ref, nccl_out, ref_fused, lout, eroutes, rroutes
            for _ in range(3):
                nstep()
            torch.cuda.synchronize()
            barrier(world)
            nt = time_steps(nstep, max(5, min(args.steps, 30)), flush, lead_cycles=LEAD)
            nccl_ms = all_max(world, sum(nt) / len(nt))
            mstep = lambda: omni_moe_ep_fused(mx, None, shard, ecomm, MOE_K, recv_cap=cap,  # noqa: E731
                                              workspace=ews, out=eout, router_weight=wr)
        else:
            mstep = lambda: clefq.omni_moe(mx, None, mg, mu, md, workspace=mws, router_weight=wr)   # noqa: E731
        for _ in range(3):
            mstep()
        torch.cuda.synchronize()
        clefq.status()
        barrier(world)
        mt = time_steps(mstep, max(5, min(args.steps, 30)), flush, lead_cycles=LEAD)
        clefq.status()
        mms = all_max(world, sum(mt) / len(mt))
        if world > 1:
            ecomm.close()
        ops = 2.0 * MOE_T * MOE_K * (MOE_H * 2 * MOE_I + MOE_I * MOE_H)
        if world > 1:
            rec_b = clefq.lib().clefq_moe_ep_record_bytes(MOE_H)
            link = (world - 1) / world * MOE_T * MOE_K * (rec_b + 2 * MOE_H)   # records out, products back
            target = max(ops / (i8_peak * 1e12), link / 770e9) * 1e3
            moe_roof = {"target_ms": target, "frac": target / mms, "int_ops_per_rank": ops,
                        "nvlink_bytes_per_rank": link}
        else:
            # the whole layer against the int8 tensor peak (its GEMMs are 0.62 T int ops), and
            # the dominant launch -- the grouped gate|up expert GEMM -- timed alone below
            moe_roof = {"bound": "tensor", "kernel": "the whole clefq_moe layer (7 launches, router linear fused "
                                                  "with the router)",
                        "achieved": ops / (mms / 1000) / 1e12, "peak": i8_peak, "unit": "TOP/s",
                        "frac": ops / (mms / 1000) / 1e12 / i8_peak, "algorithmic_ops": ops,
                        "traffic": traffic_tab.get("moe_c4_layer", {}).get("traffic_bytes")}
        moe = {"workload": "C4 Omni INT4 MoE layer: 8192 tokens per GPU, hidden 2048, 128 experts x (gate|up "
                           "2048->2x768, down 768->2048), top-8", "roofline": moe_roof,
               "parallelism": f"ep{world}: experts sharded; one clefq_moe_ep_layer call, dispatch and return "
                              "stored into peers' buffers over NVLink by the kernels" if world > 1
               else "single GPU", "tokens_per_s": world * MOE_T / (mms / 1000), "ms_per_step": mms,
               "nccl_all_to_all_ms_per_step": nccl_ms,
               "parity": parity, "parity_paths": parity_paths,
               "router": "router linear fused with the router (clefq_route_linear's kernel) inside the timed "
                         "layer; the NCCL composition routes from precomputed logits",
               "parity_note": "each rank's fused and NCCL expert-parallel outputs equal clefq_moe over the same "
                              "tokens with all 128 experts on one GPU, bit for bit (all ranks)" if world > 1 else
                              "tests/test_gpu_fullsize.py checks this layer at full size against the CPU oracle",
               "tops": ops / (mms / 1000) / 1e12, "frac_of_int8_peak": ops / (mms / 1000) / 1e12 / i8_peak}
        del mg, mu, md, mws

    # ---- tensor-parallel C2 block (N > 1): one 4096-token block shared by all ranks -------
    tp = None
    if world > 1 and not args.skip_tp:
        from clefq.tp import TpComm, mlp_tp, mlp_tp_fused, shard_mlp, tp_mlp_region_bytes
        tgen = torch.Generator(device="cuda")
        tgen.manual_seed(77)                    # the same input and weights on every rank
        tx = torch.randn(M, HIDDEN, device="cuda", generator=tgen).to(torch.bfloat16)
        tg, tu, td = (rand_weight_dev(clefq, INTER, HIDDEN, tgen), rand_weight_dev(clefq, INTER, HIDDEN, tgen),
                      rand_weight_dev(clefq, HIDDEN, INTER, tgen))
        tshard = shard_mlp(tg, tu, td, rank, world)
        comm = TpComm(tp_mlp_region_bytes(M, HIDDEN, INTER, world))
        tws = torch.empty(clefq.lib().clefq_tp_mlp_workspace_size(M, HIDDEN, INTER, world), dtype=torch.uint8,
                          device="cuda")
        tout = torch.empty((M, HIDDEN), dtype=torch.bfloat16, device="cuda")
        # parity before timing: both tensor-parallel paths against clefq_mlp on one GPU
        tref = clefq.mlp(tx, tg, tu, td)
        nccl_out = mlp_tp(tx, tshard)
        mlp_tp_fused(tx, tshard, comm, workspace=tws, out=tout)
        torch.cuda.synchronize()
        clefq.status()
        tp_parity = all_min(world, torch.equal(tout.view(torch.int16), tref.view(torch.int16)) and
                            torch.equal(nccl_out.view(torch.int16), tref.view(torch.int16)))
        del tref, nccl_out

        def timed(step):
            for _ in range(3):
                step()
            torch.cuda.synchronize()
            clefq.status()
            barrier(world)
            tt = time_steps(step, max(5, min(args.steps, 30)), flush, lead_cycles=LEAD)
            clefq.status()
            return all_max(world, sum(tt) / len(tt))
        fms = timed(lambda: mlp_tp_fused(tx, tshard, comm, workspace=tws, out=tout))
        nms = timed(lambda: mlp_tp(tx, tshard))
        barrier(world)
        comm.close()
        # fused compute+collective roofline: the slower of (int ops / int8 peak) and (bytes this
        # rank must put on NVLink / the measured 770 GB/s per direction)
        tp_ops = 2.0 * M * HIDDEN * INTER * 3 / world
        tp_link = (world - 1) * (M * (INTER // world) // 2 + M * (HIDDEN // world) * 2 + M * 4)
        tp_target = max(tp_ops / (i8_peak * 1e12), tp_link / 770e9) * 1e3
        tp = {"workload": "C2 dense INT4 SwiGLU MLP block, 4096 tokens shared by all ranks",
              "roofline": {"target_ms": tp_target, "frac": tp_target / fms, "int_ops_per_rank": tp_ops,
                           "nvlink_bytes_per_rank": tp_link, "peaks": f"{i8_peak:.0f} TOP/s int8 (2 x measured "
                           "bf16), 770 GB/s NVLink per direction (measured peer copy)"},
              "parallelism": f"tp{world}: intermediate sharded; one clefq_tp_mlp call whose packing kernel and "
                             "down-GEMM epilogue store their shards into every rank's buffer over NVLink, with "
                             "device barriers", "scaling": "strong",
              "tokens_per_s": M / (fms / 1000), "ms_per_step": fms,
              "nccl_collectives_ms_per_step": nms,
              "parity": tp_parity,
              "parity_note": "every rank's fused and NCCL tensor-parallel outputs equal clefq_mlp on one GPU "
                             "with the full weights, bit for bit",
              "gpu_launches_per_step": 8}
        del tg, tu, td

    # ---- C1: one 128 x 2048 -> 768 projection, GPU and CPU ---------
    c1 = None
    if not args.skip_c1:
        c1 = run_c1(clefq, gen, flush, args, world, rank, i8_peak)
    c3 = None if args.skip_c3 else run_c3(clefq, gen, flush, args, world, rank, i8_peak)
    c5 = None if args.skip_c5 else run_c5(clefq, gen, flush, args, world, rank, i8_peak)

    launches = 4 * args.steps
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 x int4 -> int32 (tcgen05 kind::i8), f32 epilogue, bf16 activations",
        "data": "synthetic (seed 1000+rank): x bf16 N(0,1), codes uniform [-8,7], scales |N(0,0.02)|/7",
        "config": run_config(world),
        "roofline": {"bound": "tensor",
                     "kernel": "gemm_i4_2sm_deep_kernel<dense, 256> (C2 gate|up GEMM as clefq_mlp launches it: "
                               "M=4096, N=2x12288 over two weight maps, K=4096, SwiGLU epilogue)",
                     "achieved": gu_achieved, "peak": i8_peak, "unit": "TOP/s", "frac": gu_achieved / i8_peak,
                     "traffic": traffic_tab.get("gemm_c2_gate_up", {}).get("traffic_bytes"),
                     "algorithmic_ops": gu_ops,
                     "peak_note": f"kind::i8 dense = 2 x {peak_kind} bf16 burst ({bf16_peak} TF/s) from "
                                  "MEASURED_PEAKS.json"},
        "roofline_down": {"bound": "tensor",
                          "kernel": "gemm_i4_2sm_deep_kernel<dense, 256> (C2 down GEMM M=4096 N=4096 K=12288)",
                          "achieved": down_achieved, "peak": i8_peak, "unit": "TOP/s",
                          "frac": down_achieved / i8_peak,
                          "traffic": traffic_tab.get("gemm_c2_down", {}).get("traffic_bytes"),
                          "algorithmic_ops": down_ops},
        "kernels_ms": ktimes,
        "e2e": {"value": world * M / (e2e_ms / 1000), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "api": "clefq.mlp_host (clefq_mlp_host), pinned host buffers, calls back to back",
                "chunk_rows": e2e_chunk, "steps": e2e_steps,
                "h2d_bytes_per_step": int(x.numel() * 2), "d2h_bytes_per_step": int(M * HIDDEN * 2)},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if c1:
        line["c1"] = c1
    if c3:
        line["c3"] = c3
    if c5:
        line["c5"] = c5
    if moe:
        line["secondary"] = moe
    if tp:
        line["tensor_parallel"] = tp
    if rank == 0 and world == 1 and not args.skip_cpu:
        threads = len(os.sched_getaffinity(0))
        cpu_val, reps, el = cpu_mlp_sample(512, 10.0, threads)
        line["cpu_baseline"] = {"value": cpu_val, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"{reps} x 512 of the C2 tokens through the full-size weights "
                                          f"({el:.1f} s), CPU oracle port (OpenMP, AVX-512 VNNI dot)"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="clefq", choices=["clefq", "reference"])
    ap.add_argument("--skip-moe", action="store_true")
    ap.add_argument("--skip-tp", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-c1", action="store_true")
    ap.add_argument("--skip-c3", action="store_true")
    ap.add_argument("--skip-c5", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=0,
                    help="calls in the timed e2e stream (default: --steps clamped to [100, 200]); "
                         "small values keep profiler captures short")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        # The reference arm runs on the host cores of rank 0; other ranks exit without work.
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), 0)
        return
    world, rank, local = dist_init()
    try:
        run_clefq(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
