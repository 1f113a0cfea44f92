"""Benchmark of the ternary hot path (one JSON line on stdout from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (BASELINE.json config 0/1, the metric's "ternary GEMV HBM GB/s"):
dense ternary GEMV, x f32 [1, 2048] ~ N(0,1), W [5632, 2048] ternary with
P(-1)=P(0)=P(+1)=1/3 packed in the reference's 2-bit layout, per-row scales
~ U(0.01, 0.1).  One STEP = one grouped launch of 64 such GEMVs over 64
distinct weight copies reading the same token x (the independent projections
of one decode step).  The K timed steps rotate over 128 weight copies
(352 MiB, more than 2x the 126 MB L2; every launch reads 188 MB), so each step
streams its weights from HBM.  Inputs are made on the device from a seeded
generator (synthetic data; no dataset exists for this path).

value: algorithmic GB/s over all ranks = K * 64 * 2,936,832 B * ranks / max
over ranks of the device time of the K timed steps (CUDA events on the
launching stream; the K launches replayed from one CUDA graph).

The same line carries, as sub-objects, the other BASELINE configs timed in
the same run: gemm_cfg2 (int8 prefill GEMM), sparse_cfg3 (2:4 sparse, M=1
and M=64), kv_cfg5 (3-bit KV flash decode) -- on one GPU -- and moe_cfg4
(the MoE layer, expert-parallel over all ranks, with per-phase times and a
parity check of sampled tokens against the CPU oracle) at every N.

Multi-GPU: the GEMV does not shard; each rank runs its own replica stream
(weak scaling, no collective on the data path).  The MoE layer shards its
experts over the ranks (strong scaling: the 4096-token batch is fixed).

--impl reference times the reference's CPU algorithm for the headline
workload: the C restatement of ternary_matmul_packed_parallel
(src/model/ternary.rs:471-529) with per-row scales, on all host cores (the
reference itself is Rust and cannot be built on this image; see oracle/).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

ROWS, COLS = 5632, 2048
ALGO_BYTES = ROWS * COLS // 4 + ROWS * 4 + COLS * 4 + ROWS * 4  # W + scales + x + y
GROUP = 64  # GEMVs per launch (one step)
N_COPIES = 128
METRIC = "ternary GEMV HBM GB/s"
UNIT = "GB/s"
L2_BYTES = 126 * 1024 * 1024


def load_peaks():
    """(HBM GB/s, bf16 burst TFLOP/s, source) from MEASURED_PEAKS.json, else the fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        return json.load(open(p))
    except Exception:
        return {}


def _scaled_traffic(key, factor):
    v = load_traffic().get(key, {}).get("dram_bytes_per_launch")
    return None if v is None else int(v * factor)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.dev)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.1)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxs.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sms) if sms else None,
                "sm_max_mhz": max(maxs) if maxs else None, "reasons": sorted(reasons),
                "samples": len(sms)}


class Timer:
    """Device time of work issued on `stream`, max over ranks (CUDA events,
    a barrier and a synchronize on both sides).  A ~100 us spin kernel runs on
    the stream just before the start event, outside the timed region: the GPU
    is then still busy while the host submits the first timed launch, so the
    host's submission latency (tens of us for a graph launch, 4% of a 20-step
    GEMV region) is not counted as device time."""

    LEAD_IN_CYCLES = 200_000

    def __init__(self, torch, dist, stream, device, ws):
        self.torch, self.dist, self.stream, self.device, self.ws = torch, dist, stream, device, ws

    def __call__(self, fn):
        torch = self.torch
        torch.cuda.synchronize()
        if self.ws > 1:
            self.dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            if hasattr(torch.cuda, "_sleep"):
                torch.cuda._sleep(self.LEAD_IN_CYCLES)
            e0.record(self.stream)
            fn()
            e1.record(self.stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=self.device, dtype=torch.float64)
        if self.ws > 1:
            self.dist.barrier()
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def _graph_of(torch, stream, fns):
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for f in fns:
            f()
    return graph


def _upload_u32(gpu, torch, ctx, words, rows, cols, scales, device):
    import ctypes as C

    from ferrisres_b200._lib import call
    h = C.c_void_p()
    call("ft_weight_from_device_u32", ctx.handle, C.c_void_p(words.data_ptr()), rows, cols,
         C.c_void_p(scales.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream),
         C.byref(h))
    torch.cuda.synchronize()
    return gpu.DeviceTernaryWeight(h, rows, cols, ctx)


def _words_from_codes(torch, codes):
    """codes int64 {0,1,2} [n] (n % 16 == 0) -> u32 words, 16 codes per word LSB first."""
    words = (codes.view(-1, 16) << torch.arange(0, 32, 2, device=codes.device)).sum(dim=1)
    return torch.where(words >= 2**31, words - 2**32, words).to(torch.int32).contiguous()


# --------------------------------------------------------------- headline --
def make_weights(gpu, torch, n_copies, device):
    """n_copies ternary [ROWS, COLS] matrices (P = 1/3 each) with row scales, made on the device."""
    weights = []
    g = torch.Generator(device=device)
    ctx = gpu.get_context(device.index)
    for i in range(n_copies):
        g.manual_seed(i)
        codes = torch.randint(0, 3, (ROWS * COLS,), generator=g, device=device, dtype=torch.int64)
        scales = (torch.rand(ROWS, generator=g, device=device) * 0.09 + 0.01).contiguous()
        weights.append(_upload_u32(gpu, torch, ctx, _words_from_codes(torch, codes), ROWS, COLS,
                                   scales, device))
        del codes
    return weights


def run_gemv(args, ws, rank, local, torch, dist, device):
    from ferrisres_b200 import _lib, gpu

    weights = make_weights(gpu, torch, N_COPIES, device)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    x = torch.randn(1, COLS, generator=g, device=device)
    ys = [torch.empty(1, ROWS, device=device) for _ in range(N_COPIES)]
    calls = [gpu.GroupCall(weights[i:i + GROUP], [x] * GROUP, ys[i:i + GROUP])
             for i in range(0, N_COPIES, GROUP)]
    singles = [gpu.GroupCall([weights[i]], [x], [ys[i]]) for i in range(N_COPIES)]
    stream = torch.cuda.Stream(device=device)
    timer = Timer(torch, dist, stream, device, ws)
    with torch.cuda.stream(stream):  # warm-up (also sizes workspaces before capture)
        for i in range(max(args.warmup, 3)):
            calls[i % len(calls)]()
        for i in range(3):
            singles[i]()
    stream.synchronize()

    # the K timed steps: K grouped launches, rotating over the weight copies,
    # replayed from CUDA graphs of at most 256 launches
    steps = args.steps
    chunk = min(steps, 256)
    launches0 = _lib.lib().ft_launch_counter()
    g_main = _graph_of(torch, stream, [calls[i % len(calls)] for i in range(chunk)])
    reps, rem = divmod(steps, chunk)
    g_rem = _graph_of(torch, stream, [calls[i % len(calls)] for i in range(rem)]) if rem else None
    captured = _lib.lib().ft_launch_counter() - launches0
    assert captured == chunk + rem, (captured, chunk, rem)  # one kernel launch per step
    gpu_launches = reps * chunk + rem
    with torch.cuda.stream(stream):  # warm both graphs
        g_main.replay()
        if g_rem is not None:
            g_rem.replay()

    def timed_steps():
        for _ in range(reps):
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()

    sampler = ClockSampler(local)
    sampler.start()
    sec = timer(timed_steps)
    clocks = sampler.stop()
    launch_s = sec / steps
    value = ws * steps * GROUP * ALGO_BYTES / sec / 1e9
    achieved = GROUP * ALGO_BYTES / launch_s / 1e9

    # the same GEMVs, 16 per launch, one sweep of the copies per replay
    calls16 = [gpu.GroupCall(weights[i:i + 16], [x] * 16, ys[i:i + 16])
               for i in range(0, N_COPIES, 16)]
    g16 = _graph_of(torch, stream, calls16)
    with torch.cuda.stream(stream):
        g16.replay()
    ms16 = timer(lambda: [g16.replay() for _ in range(5)])
    l16 = ms16 / (5 * len(calls16))
    del g16
    # dependent chain: each GEMV its own launch, back to back
    g_chain = _graph_of(torch, stream, singles)
    with torch.cuda.stream(stream):
        g_chain.replay()
    s_chain = timer(lambda: [g_chain.replay() for _ in range(5)]) / (5 * N_COPIES)
    del g_chain

    # end to end through the host-buffer accelerator call: pinned x in, y out
    acc = gpu.GpuMatmulAccelerator(local)
    xh = torch.empty(COLS, dtype=torch.float32, pin_memory=True)
    xh.copy_(x.view(-1).cpu())
    xn = xh.numpy()
    for i in range(5):
        acc.gpu_ternary_matmul_vram(weights[i], xn, 1, COLS, ROWS)
    n_e2e = max(64, min(steps * GROUP, 4096))
    if ws > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        acc.gpu_ternary_matmul_vram(weights[i % N_COPIES], xn, 1, COLS, ROWS)
    e2e_local = torch.tensor([(time.perf_counter() - t0) / n_e2e], device=device,
                             dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(e2e_local, op=dist.ReduceOp.MAX)
    e2e_value = ws * ALGO_BYTES / float(e2e_local.item()) / 1e9

    peak, _, peak_kind = load_peaks()
    tr = load_traffic().get("gemv_cfg1_g64", {})
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws,
        "steps": steps, "warmup": args.warmup, "ms_per_step": launch_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": "cfg1 dense ternary GEMV x f32 [1,2048] . W [5632,2048]^T, "
                               "per-row scales; one step = one launch of 64 GEMVs",
                   "rows": ROWS, "cols": COLS, "seq": 1, "gemvs_per_step": GROUP,
                   "weight_copies": N_COPIES,
                   "l2": f"inputs larger than L2: a step reads {GROUP * ROWS * COLS // 4 / 1e6:.0f} "
                         f"MB of weights; steps rotate over {N_COPIES} copies "
                         f"({N_COPIES * ROWS * COLS // 4 / 2**20:.0f} MiB)",
                   "parallelism": f"replicas x{ws}", "graph": "CUDA graph replay"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": tr.get("dram_bytes_per_launch"),
                     "traffic_source": tr.get("source"),
                     "kernel": tr.get("kernel", "gemv_kernel<1, 64, false>"),
                     "algorithmic_bytes_per_launch": GROUP * ALGO_BYTES,
                     "note": f"the timed launch: {GROUP} GEMVs of 2,936,832 algorithmic bytes "
                             "each; achieved = those bytes / the launch's average device time "
                             "(CUDA events over the K timed launches)"},
        "launch_of_16": {"GBps": round(16 * ALGO_BYTES / l16 / 1e9, 2),
                         "frac": round(16 * ALGO_BYTES / l16 / 1e9 / peak, 4),
                         "us_per_launch": round(l16 * 1e6, 3)},
        "single_gemv_chain": {"us_per_gemv": round(s_chain * 1e6, 3),
                              "GBps": round(ALGO_BYTES / s_chain / 1e9, 2),
                              "frac": round(ALGO_BYTES / s_chain / 1e9 / peak, 4),
                              "note": "each GEMV its own launch, back to back in a CUDA graph "
                                      "with programmatic dependent launch"},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": GROUP * COLS * 4,
                "d2h_bytes_per_step": GROUP * ROWS * 4, "calls": n_e2e,
                "us_per_gemv_call": round(float(e2e_local.item()) * 1e6, 2),
                "api": "ft_gpu_ternary_matmul_vram (GpuMatmulAccelerator::gpu_ternary_matmul_vram), "
                       "one synchronous call per GEMV: pinned host x in, host y out"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks,
    }
    del g_main, g_rem
    for w in weights:
        w.close()
    return res


# ------------------------------------------------------------- CPU side --
def cpu_setup():
    from oracle import oracle as fo
    rng = np.random.default_rng(0)
    t = rng.integers(-1, 2, size=ROWS * COLS).astype(np.int8)
    packed = fo.pack_ternary(t)
    rs = rng.uniform(0.01, 0.1, ROWS).astype(np.float32)
    x = rng.standard_normal(COLS).astype(np.float32)
    # the GPU arm's rotation: N_COPIES separate copies of the weights (352 MiB),
    # so the timed GEMVs stream them from memory rather than from the last-level cache
    copies = [packed.copy() for _ in range(N_COPIES)]
    return fo, copies, rs, x


def cpu_gemv_step(fo, copies, rs, x, step, threads):
    """One headline step on the CPU: GROUP GEMVs over consecutive weight copies."""
    for j in range(GROUP):
        fo.ternary_matmul_packed_parallel_rows(copies[(step * GROUP + j) % N_COPIES], rs, x, ROWS,
                                               COLS, threads)


def cpu_baseline(seconds):
    """Oracle restatement of ternary_matmul_packed_parallel timed on all host cores."""
    fo, copies, rs, x = cpu_setup()
    threads = fo.num_threads(0)
    cpu_gemv_step(fo, copies, rs, x, 0, threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_gemv_step(fo, copies, rs, x, n, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    return {"value": round(n * GROUP * ALGO_BYTES / el / 1e9, 3), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{n} steps of {GROUP} GEMVs [5632x2048] in {el:.1f} s "
                      f"(ternary_matmul_packed_parallel, per-row scales, 32 row batches over "
                      f"{threads} threads; weights rotated over {N_COPIES} copies, 352 MiB, as "
                      "in the GPU arm)"}


def run_reference(args, ws, rank):
    if rank != 0:
        return None
    fo, copies, rs, x = cpu_setup()
    threads = fo.num_threads(0)
    for i in range(min(args.warmup, 3)):
        cpu_gemv_step(fo, copies, rs, x, i, threads)
    # bounded sample: at most 60 s of CPU work, whatever --steps asks
    steps, t0 = 0, time.perf_counter()
    while steps < args.steps:
        cpu_gemv_step(fo, copies, rs, x, steps, threads)
        steps += 1
        if time.perf_counter() - t0 > 60.0:
            break
    el = time.perf_counter() - t0
    value = steps * GROUP * ALGO_BYTES / el / 1e9
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": ws, "steps": steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": "cfg1 dense ternary GEMV x f32 [1,2048] . W [5632,2048]^T, "
                               "per-row scales; one step = 64 GEMVs",
                   "rows": ROWS, "cols": COLS, "seq": 1, "gemvs_per_step": GROUP,
                   "weight_copies": N_COPIES},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{steps} steps of {GROUP} GEMVs (requested {args.steps}; "
                                   "capped at 60 s); C restatement of "
                                   "ternary_matmul_packed_parallel, src/model/ternary.rs:471-529, "
                                   f"on a persistent pool of {threads} threads; weights rotated "
                                   f"over {N_COPIES} copies (352 MiB), as in the GPU arm"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------- cfg2 GEMM --
G_M, G_K, G_N = 512, 4096, 11008
G_OPS = 2 * G_M * G_K * G_N


def run_gemm(args, torch, dist, device, local, sub_steps, cpu_seconds):
    """int8 prefill GEMM (bf16 x -> per-token absmax int8 ->
    exact int32 ternary matmul -> f32), W [11008, 4096] with P(0)=0.5.  One step
    = quantize + matmul; weights rotate over copies totalling > 2x L2."""
    from ferrisres_b200 import _lib, gpu

    n_copies = max(3, -(-2 * L2_BYTES // (G_N * G_K // 4)))
    weights = []
    g = torch.Generator(device=device)
    ctx = gpu.get_context(local)
    for i in range(n_copies):
        g.manual_seed(100 + i)
        u = torch.rand(G_N * G_K, generator=g, device=device)
        codes = torch.where(u < 0.25, 0, torch.where(u < 0.75, 1, 2)).to(torch.int64)
        scales = (torch.rand(G_N, generator=g, device=device) * 0.09 + 0.01).contiguous()
        weights.append(_upload_u32(gpu, torch, ctx, _words_from_codes(torch, codes), G_N, G_K,
                                   scales, device))
        del u, codes
    g.manual_seed(7)
    xb = torch.randn(G_M, G_K, generator=g, device=device).to(torch.bfloat16)
    y = torch.empty(G_M, G_N, device=device)
    q = torch.empty(G_M, G_K, dtype=torch.int8, device=device)
    sx = torch.empty(G_M, dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device=device)
    timer = Timer(torch, dist, stream, device, 1)
    import ctypes as C

    from ferrisres_b200._lib import call

    def step(i, quant=True):
        s = C.c_void_p(stream.cuda_stream)
        if quant:
            call("ft_quantize_absmax_i8_bf16", ctx.handle, G_M, G_K, C.c_void_p(xb.data_ptr()),
                 C.c_void_p(q.data_ptr()), C.c_void_p(sx.data_ptr()), s)
        call("ft_ternary_matmul_i8", ctx.handle, weights[i % n_copies].handle, G_M,
             C.c_void_p(q.data_ptr()), C.c_void_p(sx.data_ptr()), C.c_void_p(y.data_ptr()), s)

    for i in range(3):
        step(i)
    stream.synchronize()
    launches0 = _lib.lib().ft_launch_counter()
    step(0)
    per_step = _lib.lib().ft_launch_counter() - launches0
    stream.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    sec = timer(lambda: [step(i) for i in range(sub_steps)]) / sub_steps
    clocks = sampler.stop()
    mm = timer(lambda: [step(i, False) for i in range(sub_steps)]) / sub_steps
    _, bf16, kind = load_peaks()
    peak = 2 * bf16
    tops = G_OPS / sec / 1e12
    res = {
        "metric": "ternary int8 prefill GEMM TOPS", "value": round(tops, 2), "unit": "TOPS",
        "steps": sub_steps, "ms_per_step": sec * 1e3, "dtype": "int8",
        "config": {"workload": "cfg2 prefill GEMM M=512 K=4096 N=11008, bf16 x -> absmax int8",
                   "weight_copies": n_copies, "l2": "weights rotate over copies > 2x L2"},
        "roofline": {"bound": "tensor", "achieved": round(G_OPS / mm / 1e12, 2),
                     "peak": round(peak, 1), "unit": "TOP/s",
                     "frac": round(G_OPS / mm / 1e12 / peak, 4),
                     "peak_source": f"2 x {kind} bf16 dense burst (int8 dense rate is twice "
                                    "bf16 on B200)",
                     "traffic": load_traffic().get("gemm_cfg2", {}).get("dram_bytes_per_launch"),
                     "kernel": "tq_grouped_kernel<128, false> (+ prep_b_kernel)",
                     "ms_matmul": round(mm * 1e3, 4),
                     "note": "achieved = int ops / device time of the matmul call alone "
                             "(prep + tensor-core kernel); value includes the quantizer"},
        "step_frac": round(tops / peak, 4),
        "gpu_launches": int(per_step * sub_steps),
        "clocks": clocks,
    }
    for w in weights:
        w.close()
    if cpu_seconds > 0:
        res["cpu_baseline"] = gemm_cpu_baseline(cpu_seconds)
    return res


def run_midm(args, torch, dist, device, local, sub_steps, cpu_seconds):
    """Mid-size activations on the cfg2 weight shape W[11008, 4096]: device time per matmul
    call at each M (int8 and fp32 activations), CUDA-graph replay of 12 calls over 12
    weight copies (135 MB > L2).  Covers the shapes between the decode GEMV (<= 16
    activation columns) and the wide tensor-core passes (>= 128 columns), where the
    engine's K-split choice decides the time.  Not part of the default line."""
    from ferrisres_b200 import gpu
    ctx = gpu.get_context(local)
    g = torch.Generator(device=device)
    weights = []
    for i in range(12):
        g.manual_seed(100 + i)
        u = torch.rand(G_N * G_K, generator=g, device=device)
        codes = torch.where(u < 0.25, 0, torch.where(u < 0.75, 1, 2)).to(torch.int64)
        scales = (torch.rand(G_N, generator=g, device=device) * 0.09 + 0.01).contiguous()
        weights.append(_upload_u32(gpu, torch, ctx, _words_from_codes(torch, codes), G_N, G_K,
                                   scales, device))
        del u, codes
    stream = torch.cuda.Stream(device=device)

    def graph_us(fn, reps=8):
        with torch.cuda.stream(stream):
            for i in range(12):
                fn(i)  # grows the workspaces before capture
            stream.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for i in range(12):
                    fn(i)
            for _ in range(2):
                gr.replay()
            stream.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                gr.replay()
            e1.record(stream)
            stream.synchronize()
        del gr
        return e0.elapsed_time(e1) / (reps * 12) * 1e3

    wbytes = G_N * G_K // 4
    rows = []
    gen = torch.Generator(device=device)
    gen.manual_seed(3)
    for kind, ms in (("int8", (8, 16, 17, 24, 32, 48, 64, 96, 128, 256, 512)),
                     ("fp32", (2, 3, 4, 8, 12, 16, 32, 64))):
        for m in ms:
            y = torch.empty(m, G_N, device=device)
            if kind == "int8":
                q = torch.randint(-127, 128, (m, G_K), dtype=torch.int8, device=device,
                                  generator=gen)
                sx = torch.rand(m, device=device, generator=gen) * 0.01
                us = graph_us(lambda i: weights[i % 12].matmul_i8(q, sx, out=y, stream=stream))
            else:
                x = torch.randn(m, G_K, device=device, generator=gen)
                us = graph_us(lambda i: weights[i % 12].matmul_f32(x, out=y, stream=stream))
            rows.append({"act": kind, "M": m, "us": round(us, 2),
                         "weight_GBps": round(wbytes / us / 1e3, 1),
                         "TOPS": round(2 * m * G_N * G_K / us / 1e6, 1)})
    for w in weights:
        w.close()
    return {"metric": "mid-size M ternary matmul time", "unit": "us per call",
            "config": {"workload": "W[11008, 4096], M = 2..512, 12 weight copies > L2, "
                                   "CUDA-graph replay"},
            "rows": rows}


def gemm_cpu_baseline(seconds):
    """Oracle restatement of ternary_matmul_parallel (over tokens) on int8 codes as f32,
    on all host cores, over a bounded sample of the 512 tokens."""
    from oracle import oracle as fo
    rng = np.random.default_rng(0)
    t = rng.choice(np.array([-1, 0, 1], np.int8), size=G_N * G_K, p=[0.25, 0.5, 0.25])
    sw = rng.uniform(0.01, 0.1, G_N).astype(np.float32)
    tok = 32
    x = rng.standard_normal((tok, G_K)).astype(np.float32)
    qx, sxs = fo.quantize_absmax_i8(x.ravel(), tok, G_K)
    threads = fo.num_threads(0)
    n, t0 = 0, time.perf_counter()
    while True:
        fo.ternary_matmul_i8(t, qx, sxs, sw, tok, G_K, G_N, threads, via_f32=True)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 2:
            break
    ops = n * 2 * tok * G_K * G_N
    return {"value": round(ops / el / 1e12, 5), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{n} x {tok} of the 512 tokens in {el:.1f} s (ternary_matmul_parallel on "
                      "the int8 codes as f32, src/model/ternary.rs:333-389, parallel over tokens)"}


# ------------------------------------------------------------ cfg3 2:4 ---
S_N, S_K = 14336, 4096
S_GROUP, S_COPIES = 32, 64


def run_sparse(args, torch, dist, device, local, sub_steps, cpu_seconds):
    """2:4 sparse ternary matmul, K=4096, N=14336, fp32 x,
    at M=1 (decode GEMV kernel; one step = one launch of 32 GEMVs over distinct
    weight copies) and M=64 (tensor-core engine).  Weights enter in the
    reference SparseTernaryMatrix layout and are stored at 1.5 bits/weight
    (the sparse MMA's metadata nibble + two sign bits per group of 4, the size
    of the reference's own packing); copies rotate beyond 2x L2."""
    from ferrisres_b200 import gpu

    dev_bytes = (S_N // 128) * (S_K // 128) * 3072
    algo = dev_bytes + S_N * 4 + S_K * 4 + S_N * 4  # weights + scales + x + y per GEMV
    rng = np.random.default_rng(0)
    ng = S_N * S_K // 4
    weights = []
    for i in range(S_COPIES):
        if i < 4:  # 4 distinct matrices, uploaded as separate copies beyond that
            lo = rng.integers(0, 6, size=(ng + 1) // 2, dtype=np.uint8)
            hi = rng.integers(0, 6, size=(ng + 1) // 2, dtype=np.uint8)
            pat = (lo | (hi << 4)).astype(np.uint8)
            sg = rng.integers(0, 256, size=(ng + 3) // 4, dtype=np.uint8)
            rs = rng.uniform(0.01, 0.1, S_N).astype(np.float32)
        weights.append(gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, S_N, S_K, rs, local))
    assert weights[0].device_bytes() == dev_bytes + S_N * 4
    x1 = torch.randn(1, S_K, device=device)
    x64 = torch.randn(64, S_K, device=device)
    ys = [torch.empty(1, S_N, device=device) for _ in range(S_COPIES)]
    y64 = torch.empty(64, S_N, device=device)
    calls = [gpu.GroupCall(weights[i:i + S_GROUP], [x1] * S_GROUP, ys[i:i + S_GROUP])
             for i in range(0, S_COPIES, S_GROUP)]
    stream = torch.cuda.Stream(device=device)
    timer = Timer(torch, dist, stream, device, 1)
    with torch.cuda.stream(stream):
        for c in calls:
            c()
        weights[0].matmul_f32(x64, out=y64)
    stream.synchronize()
    graph = _graph_of(torch, stream, [calls[i % len(calls)] for i in range(sub_steps)])
    with torch.cuda.stream(stream):
        graph.replay()
    sampler = ClockSampler(local)
    sampler.start()
    sec = timer(graph.replay) / sub_steps
    clocks = sampler.stop()
    gbps = S_GROUP * algo / sec / 1e9

    def m64():
        for i in range(sub_steps):
            weights[i % S_COPIES].matmul_f32(x64, out=y64)
    with torch.cuda.stream(stream):
        m64()
    sec64 = timer(lambda: m64()) / sub_steps
    peak, _, kind = load_peaks()
    del graph
    for w in weights:
        w.close()
    res = {
        "metric": "2:4 sparse ternary GEMV HBM GB/s", "value": round(gbps, 2), "unit": "GB/s",
        "steps": sub_steps, "ms_per_step": sec * 1e3, "dtype": "f32",
        "config": {"workload": "cfg3 2:4 sparse K=4096 N=14336, M=1 (one step = one launch of "
                               f"{S_GROUP} GEMVs) and M=64", "device_bytes_per_weight": dev_bytes,
                   "bits_per_weight": 1.5, "weight_copies": S_COPIES,
                   "l2": f"a step reads {S_GROUP * dev_bytes / 1e6:.0f} MB of weights (> L2)"},
        "roofline": {"bound": "hbm", "achieved": round(gbps, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(gbps / peak, 4), "peak_source": kind,
                     "algorithmic_bytes_per_launch": S_GROUP * algo,
                     "traffic": _scaled_traffic("sparse_cfg3", 1),
                     "traffic_note": "DRAM bytes of one captured launch of the same 32 GEMVs",
                     "kernel": "gemv_kernel<1, 64, true>"},
        "m64": {"ms": round(sec64 * 1e3, 4),
                "TOPS_nonzero": round(2 * 64 * S_N * S_K / 2 / sec64 / 1e12, 2),
                "GBps_weights": round(dev_bytes / sec64 / 1e9, 1)},
        "gpu_launches": int(sub_steps),
        "clocks": clocks,
    }
    if cpu_seconds > 0:
        res["cpu_baseline"] = sparse_cpu_baseline(cpu_seconds, algo)
    return res


def sparse_cpu_baseline(seconds, algo):
    """Oracle restatement of sparse_ternary_matmul (src/model/sparse_ternary.rs:203-252),
    M=1, host layout, all host cores."""
    from oracle import oracle as fo
    rng = np.random.default_rng(0)
    ng = S_N * S_K // 4
    lo = rng.integers(0, 6, size=(ng + 1) // 2, dtype=np.uint8)
    hi = rng.integers(0, 6, size=(ng + 1) // 2, dtype=np.uint8)
    pat = (lo | (hi << 4)).astype(np.uint8)
    sg = rng.integers(0, 256, size=(ng + 3) // 4, dtype=np.uint8)
    rs = rng.uniform(0.01, 0.1, S_N).astype(np.float32)
    x = rng.standard_normal(S_K).astype(np.float32)
    threads = fo.num_threads(0)
    n, t0 = 0, time.perf_counter()
    while True:
        fo.sparse_ternary_matmul(pat, sg, 1.0, rs, S_N, S_K, x, 1, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    return {"value": round(n * algo / el / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{n} GEMVs (M=1) in {el:.1f} s; bytes counted as the GPU arm's "
                      "algorithmic bytes per GEMV"}


# ------------------------------------------------------------- cfg4 MoE ---
M_E, M_H, M_F, M_T, M_K = 64, 2048, 1408, 4096, 2
M_OPS = M_T * M_K * (3 * 2 * M_H * M_F) + 2 * M_T * M_E * M_H
M_SAMPLE = 16  # tokens of rank 0's shard checked against the oracle


def _rand_packed(rng, rows, cols):
    """Reference pack_ternary bytes of a matrix with P(-1)=P(0)=P(+1)=1/3."""
    c = rng.integers(0, 3, size=(rows * cols // 4, 4), dtype=np.uint8)
    return (c[:, 0] | (c[:, 1] << 2) | (c[:, 2] << 4) | (c[:, 3] << 6)).astype(np.uint8)


def _moe_expert(e):
    """Expert e's packed gate/up/down bytes and row scales (seeded by e; the
    same on every rank)."""
    wrng = np.random.default_rng(1000 + e)
    g = _rand_packed(wrng, M_F, M_H)
    u = _rand_packed(wrng, M_F, M_H)
    d = _rand_packed(wrng, M_H, M_F)
    gs = wrng.uniform(0.01, 0.1, M_F).astype(np.float32)
    us = wrng.uniform(0.01, 0.1, M_F).astype(np.float32)
    ds = wrng.uniform(0.01, 0.1, M_H).astype(np.float32)
    return g, u, d, gs, us, ds


def _moe_router():
    import torch
    rng = np.random.default_rng(4)
    router = (rng.standard_normal(M_E * M_H) * 0.02).astype(np.float32)
    return torch.from_numpy(router).to(torch.bfloat16).float().numpy()  # bf16 router weights


def moe_parity(x_sample, y_sample, router):
    """Checks sampled tokens of the layer output against the oracle's
    TernaryMoELayer::forward restatement (per-row scales).  Routing must agree
    except on near-ties (k-th and (k+1)-th probabilities within 1e-6); outputs
    of agreeing tokens within 1e-4 * rms(y_ref[t]) + 1e-7 per element."""
    from oracle import oracle as fo
    T = x_sample.shape[0]
    x = x_sample.astype(np.float32)
    # routing on the CPU first, to build only the experts the sample needs
    logits = (x.astype(np.float64) @ router.reshape(M_E, M_H).T.astype(np.float64))
    top = np.argsort(-logits, axis=1)[:, :M_K + 2]
    need = sorted(set(top.ravel().tolist()))
    zero_in = np.zeros(M_F * M_H, np.int8)
    zero_s_f = np.zeros(M_F, np.float32)
    zero_s_h = np.zeros(M_H, np.float32)
    g, u, d, gs, us, ds = ([zero_in] * M_E, [zero_in] * M_E, [zero_in] * M_E, [zero_s_f] * M_E,
                           [zero_s_f] * M_E, [zero_s_h] * M_E)
    g, u, d, gs, us, ds = list(g), list(u), list(d), list(gs), list(us), list(ds)
    for e in need:
        pg, pu, pd, sg, su, sd = _moe_expert(e)
        g[e] = fo.unpack_ternary(pg, M_F * M_H)
        u[e] = fo.unpack_ternary(pu, M_F * M_H)
        d[e] = fo.unpack_ternary(pd, M_H * M_F)
        gs[e], us[e], ds[e] = sg, su, sd
    ref_y, ref_route, ref_probs = fo.moe_forward(router, g, gs, u, us, d, ds, M_H, M_F, M_K,
                                                 x.ravel(), T)
    ref_y = ref_y.reshape(T, M_H).astype(np.float64)
    ref_probs = ref_probs.reshape(T, M_E)
    ref_route = ref_route.reshape(T, M_K)
    if not set(ref_route.ravel().tolist()) <= set(need):
        return {"ok": False, "why": "oracle routed to an expert outside the prepared set"}
    srt = -np.sort(-ref_probs, axis=1)
    near_tie = (srt[:, M_K - 1] - srt[:, M_K]) < 1e-6
    rms = np.sqrt(np.mean(ref_y ** 2, axis=1, keepdims=True))
    err = np.abs(y_sample.astype(np.float64) - ref_y) / (1e-4 * rms + 1e-7)
    worst_tok = err.max(axis=1)
    ok = bool(((worst_tok <= 1.0) | near_tie).all())
    return {"ok": ok, "tokens": int(T), "near_ties": int(near_tie.sum()),
            "worst_err_over_tol": round(float(worst_tok[~near_tie].max()) if (~near_tie).any()
                                        else 0.0, 4),
            "rule": "|y - y_ref| <= 1e-4 * rms(y_ref[t]) + 1e-7, near-ties excepted"}


def run_moe(args, torch, dist, device, ws, rank, local, sub_steps, cpu_seconds):
    """ternary MoE FFN layer, 64 experts, H=2048, F=1408,
    SwiGLU, top-2, 4096 bf16 tokens; expert-parallel over the ranks (rank r
    holds experts [r*64/N, (r+1)*64/N) and routes 4096/N tokens).  One step = one
    layer forward over the global batch.  value = 4096 tokens / max-over-ranks
    device time (strong scaling: the layer and batch are fixed)."""
    from ferrisres_b200 import moe, moe_ep

    router = _moe_router()
    per = M_E // ws
    mine = range(rank * per, (rank + 1) * per)
    g, u, d, gs, us, ds = [], [], [], [], [], []
    for e in range(M_E):
        if e in mine:
            pg, pu, pd, sg, su, sd = _moe_expert(e)
            g.append(pg); u.append(pu); d.append(pd); gs.append(sg); us.append(su); ds.append(sd)
        else:
            for lst in (g, u, d, gs, us, ds):
                lst.append(None)
    layer = moe.TernaryMoELayer(router, g, gs, u, us, d, ds, M_H, M_F, M_K, device=local)
    be = moe_ep.GpuMoEBackend(layer)
    gx = torch.Generator(device=device).manual_seed(99)
    x = torch.randn(M_T, M_H, generator=gx, device=device).to(torch.bfloat16)
    shard = x.chunk(ws)[rank].contiguous()
    stream = torch.cuda.Stream(device=device)
    timer = Timer(torch, dist, stream, device, ws)
    # micro-batches per step (ferrisres_b200/moe_ep.py): 1 by default -- on one
    # GPU two micro-batches cost more in launches (1.106 vs 0.994 ms per step)
    # than the host wait they hide
    micro = args.ep_micro if args.ep_micro > 0 else 1
    with torch.cuda.stream(stream):
        for _ in range(3):
            y = moe_ep.ep_forward(shard, be, M_E, rank, ws, micro=micro)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()

    def steps():
        for _ in range(sub_steps):
            moe_ep.ep_forward(shard, be, M_E, rank, ws, micro=micro)
    sec = timer(steps) / sub_steps
    clocks = sampler.stop()
    # per-phase device times of one instrumented step (max over ranks)
    marks, stats = [], {}
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    with torch.cuda.stream(stream):
        y = moe_ep.ep_forward(shard, be, M_E, rank, ws, marks=marks, stats=stats)
    torch.cuda.synchronize()
    ph = torch.tensor([marks[i - 1][1].elapsed_time(marks[i][1]) * 1e3
                       for i in range(1, len(marks))], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
    phases = {marks[i][0]: round(float(ph[i - 1]), 1) for i in range(1, len(marks))}
    nb = torch.tensor([stats.get("sent_rows_remote", 0) * M_H * 2,
                       stats.get("recv_rows_remote", 0) * M_H * 4], device=device,
                      dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(nb)
    parity = None
    if rank == 0:
        parity = moe_parity(shard[:M_SAMPLE].float().cpu().numpy(),
                            y[:M_SAMPLE].cpu().numpy(), router)
    if ws > 1:
        dist.barrier()
    res = {
        "metric": "MoE-layer tokens/s", "value": round(M_T / sec, 1), "unit": "tokens/s",
        "n_gpus": ws, "steps": sub_steps, "ms_per_step": sec * 1e3, "scaling": "strong",
        "dtype": "bf16 x, ternary experts, exact int8-digit expert GEMMs",
        "config": {"workload": "cfg4 ternary MoE FFN: 64 experts, H=2048, F=1408, SwiGLU, top-2, "
                               "4096 tokens", "parallelism": f"ep{ws}",
                   "experts_per_gpu": per, "tokens_per_gpu": M_T // ws,
                   "micro_batches": micro},
        "algorithmic_TOPS": round(M_OPS / sec / 1e12, 2),
        "phases_us": phases,
        "phases_note": "one extra step, not micro-batched, each phase closed by an event on the "
                       "stream (host gaps included); max over ranks",
        "nccl_bytes_per_step": {"dispatch": int(nb[0].item()), "combine": int(nb[1].item()),
                                "note": "rows sent to other ranks (bf16 in, fp32 out), all ranks"},
        "parity": parity,
        "clocks": clocks,
    }
    if ws == 1:
        res["decode"] = moe_decode_times(torch, layer, x, stream, timer)
    layer.close()
    if rank == 0 and ws == 1 and cpu_seconds > 0:
        res["cpu_baseline"] = moe_cpu_baseline(cpu_seconds, router)
    return res


def moe_decode_times(torch, layer, x, stream, timer):
    """Decode steps of the same layer: the fused single-launch ft_moe_decode at
    T = 1, 4, 8 tokens (replayed from a CUDA graph: the step has no host
    synchronisation), against the general ft_moe_forward at T = 1 (which reads
    the per-expert counts back to size its launches)."""
    out = {}
    reps = 50
    for T in (1, 4, 8):
        xt = x[:T].contiguous()
        with torch.cuda.stream(stream):
            layer.decode_device(xt)  # sizes the scratch before capture
        stream.synchronize()
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(reps):
                    layer.decode_device(xt)
            with torch.cuda.stream(stream):
                g.replay()
            sec = timer(g.replay) / reps
            out["graph"] = True
            del g
        except Exception as e:  # capture refused: time direct launches instead
            out["graph"] = f"not captured ({type(e).__name__})"
            torch.cuda.synchronize()

            def direct():
                for _ in range(reps):
                    layer.decode_device(xt)
            sec = timer(direct) / reps
        out[f"T{T}_us"] = round(sec * 1e6, 2)
        out[f"T{T}_us_per_token"] = round(sec * 1e6 / T, 2)
    x1 = x[:1].contiguous()

    def fwd():
        for _ in range(reps):
            layer.forward_device(x1)
    with torch.cuda.stream(stream):
        fwd()
    out["forward_T1_us"] = round(timer(fwd) / reps * 1e6, 2)
    out["note"] = ("ft_moe_decode: router, top-2, gate/up, SwiGLU, down and combine in one "
                   "cooperative launch; forward_T1: the general layer (route, layout, gather, host "
                   "read of the counts, grouped expert GEMMs, combine)")
    return out


def moe_cpu_baseline(seconds, router):
    """Oracle restatement of TernaryMoELayer::forward (per-row scales), parallel over
    tokens on all host cores, over a bounded sample of tokens."""
    from oracle import oracle as fo
    g, u, d, gs, us, ds = [], [], [], [], [], []
    for e in range(M_E):
        pg, pu, pd, sg, su, sd = _moe_expert(e)
        g.append(fo.unpack_ternary(pg, M_F * M_H)); u.append(fo.unpack_ternary(pu, M_F * M_H))
        d.append(fo.unpack_ternary(pd, M_H * M_F)); gs.append(sg); us.append(su); ds.append(sd)
    rng = np.random.default_rng(9)
    tok = 64
    x = rng.standard_normal(tok * M_H).astype(np.float32)
    threads = fo.num_threads(0)
    n, t0 = 0, time.perf_counter()
    while True:
        fo.moe_forward(router, g, gs, u, us, d, ds, M_H, M_F, M_K, x, tok, nthreads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 2:
            break
    return {"value": round(n * tok / el, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} x {tok} tokens in {el:.1f} s (TernaryMoELayer::forward restated, "
                      "src/model/ternary_moe.rs:145-223, parallel over tokens)"}


# ---------------------------------------------------------- cfg5 3-bit KV --
KV_B, KV_HQ, KV_HKV, KV_D, KV_S = 32, 32, 8, 128, 32768
KV_CACHE_BYTES = KV_B * KV_HKV * KV_S * (48 + 48 + 8 + 8)  # codes + (min, max), K and V
KV_IO_BYTES = 2 * KV_B * KV_HQ * KV_D * 4                  # q in, out
KV_ALGO_BYTES = KV_CACHE_BYTES + KV_IO_BYTES


def run_kv(args, torch, dist, device, local, sub_steps, cpu_seconds):
    """TurboQuant 3-bit KV flash decode, B=32, Hq=32, Hkv=8,
    d=128, context 32768 (reference scheme: per-vector min/max, 3-bit codes).
    One step = append one position per sequence (bf16 K, V) + evict the oldest
    (the context stays at 32768) + flash decode over the cache.  value = the
    step's algorithmic bytes (cache read + q/out) / device time."""
    from ferrisres_b200 import _lib, kv

    cache = kv.Kv3Cache(KV_B, KV_HKV, KV_S + 64, device=local)
    gen = torch.Generator(device=device).manual_seed(5)
    chunk = 4096
    for _ in range(KV_S // chunk):
        kk = torch.randn((KV_B, chunk, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
        vv = torch.randn((KV_B, chunk, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
        cache.append(kk, vv)
        del kk, vv
    q = torch.randn((KV_B, KV_HQ, KV_D), device=device, generator=gen)
    out = torch.empty_like(q)
    k1 = torch.randn((KV_B, 1, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
    v1 = torch.randn((KV_B, 1, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
    stream = torch.cuda.Stream(device=device)
    timer = Timer(torch, dist, stream, device, 1)

    def step():
        cache.append(k1, v1, stream=stream)
        cache.evict_front(1)
        cache.flash_decode(q, out=out, stream=stream)

    for _ in range(3):
        step()
    stream.synchronize()
    launches0 = _lib.lib().ft_launch_counter()
    sampler = ClockSampler(local)
    sampler.start()
    step_s = timer(lambda: [step() for _ in range(sub_steps)]) / sub_steps
    clocks = sampler.stop()
    gpu_launches = _lib.lib().ft_launch_counter() - launches0
    dec_s = timer(lambda: [cache.flash_decode(q, out=out, stream=stream)
                           for _ in range(sub_steps)]) / sub_steps
    value = KV_ALGO_BYTES / step_s / 1e9

    # end to end through the public API with host buffers: q and the new K/V
    # from pinned host memory, the output read back every step
    qh = torch.empty_like(q, device="cpu").pin_memory()
    qh.copy_(q.cpu())
    kh = torch.empty_like(k1, device="cpu").pin_memory()
    kh.copy_(k1.cpu())
    oh = torch.empty_like(out, device="cpu").pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k1), torch.empty_like(v1)

    def e2e_steps():
        for _ in range(sub_steps):
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(kh, non_blocking=True)
            cache.append(kd, vd, stream=stream)
            cache.evict_front(1)
            cache.flash_decode(qd, out=out, stream=stream)
            oh.copy_(out, non_blocking=True)
    e2e_s = timer(e2e_steps) / sub_steps
    cache.ctx.check()
    peak, _, kind = load_peaks()
    dec_gbs = KV_ALGO_BYTES / dec_s / 1e9
    cache.close()
    mode_t = kv_mode_t_times(torch, kv, device, local, timer, stream, q, out, k1, v1, sub_steps)
    paged = kv_paged_times(torch, device, local, timer, stream, q, out, sub_steps)
    res = {
        "metric": "3-bit KV flash-decode HBM GB/s", "value": round(value, 2), "unit": "GB/s",
        "steps": sub_steps, "ms_per_step": step_s * 1e3, "dtype": "u8 codes / f32",
        "config": {"workload": "cfg5 3-bit KV flash decode: B=32, Hq=32, Hkv=8, d=128, ctx 32768, "
                               "reference TurboQuantKVCache scheme (min/max per 128-vector)",
                   "step": "append 1 position + evict oldest + decode",
                   "l2": f"cache {KV_CACHE_BYTES / 2**20:.0f} MiB > L2",
                   "decode_tokens_per_s": round(KV_B / step_s, 1)},
        "roofline": {"bound": "hbm", "achieved": round(dec_gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(dec_gbs / peak, 4), "peak_source": kind,
                     "traffic": load_traffic().get("kv_cfg5", {}).get("dram_bytes_per_launch"),
                     "kernel": "kv3_decode_kernel (+ kv3_combine_kernel)",
                     "algorithmic_bytes_per_launch": KV_ALGO_BYTES,
                     "note": "112 B per (sequence, position, kv head) + q/out; decode timed alone"},
        "e2e": {"value": round(KV_ALGO_BYTES / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": q.numel() * 4 + 2 * k1.numel() * 2,
                "d2h_bytes_per_step": out.numel() * 4,
                "api": "Kv3Cache.append + flash_decode (ft_kv3_append, ft_flash_decode_3bit)"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks,
        "mode_t": mode_t,
        "paged": paged,
    }
    if cpu_seconds > 0:
        res["cpu_baseline"] = kv_cpu_baseline(cpu_seconds)
    return res


def kv_paged_times(torch, device, local, timer, stream, q, out, sub_steps):
    """The cfg5 decode through block tables: 32 requests of 32768 positions in
    a page pool (pages handed out by the PagedAttention allocator, so a
    request's pages are not contiguous), decoded by ft_kvp_flash_decode with
    the tables already on the device."""
    import ctypes as C

    from ferrisres_b200 import paged
    from ferrisres_b200._lib import call
    from ferrisres_b200.gpu import _dptr
    pages_per = KV_S // paged.PAGE_POSITIONS
    cache = paged.PagedKv3Cache(1, KV_B * pages_per + 8, KV_HKV, device=local)
    rids = [cache.create_request() for _ in range(KV_B)]
    gen = torch.Generator(device=device).manual_seed(7)
    chunk = 4096
    for _ in range(KV_S // chunk):
        kk = torch.randn((KV_B, chunk, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
        vv = torch.randn((KV_B, chunk, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
        cache.append(0, rids, kk, vv)
        del kk, vv
    tables, stride = cache._tables(0, rids)
    lens = torch.full((KV_B,), KV_S, dtype=torch.int32, device=device)

    def dec():
        call("ft_kvp_flash_decode", cache.ctx.handle, cache.handle, KV_B, _dptr(tables), stride,
             _dptr(lens), KV_S, _dptr(q), KV_HQ, C.c_float(0.0), _dptr(out),
             C.c_void_p(stream.cuda_stream))

    for _ in range(3):
        with torch.cuda.stream(stream):
            dec()
    stream.synchronize()
    dec_s = timer(lambda: [dec() for _ in range(sub_steps)]) / sub_steps
    cache.ctx.check()
    cache.close()
    peak, _, _ = load_peaks()
    gbs = KV_ALGO_BYTES / dec_s / 1e9
    return {"decode_us": round(dec_s * 1e6, 2), "decode_gbs": round(gbs, 2),
            "decode_frac": round(gbs / peak, 4),
            "note": "32 requests x 32768 positions in 32-position pages from the block "
                    "allocator; tables resident on the device"}


def kv_mode_t_times(torch, kv, device, local, timer, stream, q, out, k1, v1, sub_steps):
    """The same step and decode over a mode-T cache (rotation + uniform 3-bit
    codebook + norm): same stored bytes per position, plus the q and output
    rotations."""
    cache = kv.Kv3Cache(KV_B, KV_HKV, KV_S + 64, device=local, mode="T", seed=1)
    gen = torch.Generator(device=device).manual_seed(6)
    chunk = 4096
    for _ in range(KV_S // chunk):
        kk = torch.randn((KV_B, chunk, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
        vv = torch.randn((KV_B, chunk, KV_HKV, KV_D), device=device, generator=gen).to(torch.bfloat16)
        cache.append(kk, vv)
        del kk, vv

    def step():
        cache.append(k1, v1, stream=stream)
        cache.evict_front(1)
        cache.flash_decode(q, out=out, stream=stream)

    for _ in range(3):
        step()
    stream.synchronize()
    step_s = timer(lambda: [step() for _ in range(sub_steps)]) / sub_steps
    dec_s = timer(lambda: [cache.flash_decode(q, out=out, stream=stream)
                           for _ in range(sub_steps)]) / sub_steps
    cache.ctx.check()
    cache.close()
    peak, _, _ = load_peaks()
    gbs = KV_ALGO_BYTES / dec_s / 1e9
    return {"ms_per_step": step_s * 1e3, "value": round(KV_ALGO_BYTES / step_s / 1e9, 2),
            "decode_us": round(dec_s * 1e6, 2), "decode_gbs": round(gbs, 2),
            "decode_frac": round(gbs / peak, 4),
            "decode_tokens_per_s": round(KV_B / step_s, 1)}


def kv_cpu_baseline(seconds):
    """Oracle restatement of get_range dequant + flash_decode_ref with GQA, on all host
    cores, over a bounded sample: one sequence (of 32) at the full 32768 context."""
    from oracle import oracle as fo
    rng = np.random.default_rng(0)
    S = KV_S
    kc = rng.integers(0, 256, size=(1, S, KV_HKV * 48), dtype=np.uint8)
    vc = rng.integers(0, 256, size=(1, S, KV_HKV * 48), dtype=np.uint8)
    mn = rng.standard_normal((1, S, KV_HKV, 1)).astype(np.float32) - 2.5
    km = np.concatenate([mn, mn + 5.0], axis=-1).astype(np.float32)
    vm = km.copy()
    q = rng.standard_normal((1, KV_HQ, KV_D)).astype(np.float32)
    threads = fo.num_threads(0)
    n, t0 = 0, time.perf_counter()
    while True:
        fo.flash_decode_3bit(q, kc, km, vc, vm, 1, S, KV_HQ, KV_HKV, KV_D, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    per_seq = KV_ALGO_BYTES / KV_B
    return {"value": round(n * per_seq / el / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{n} decodes of 1 sequence x 32 q heads over 32768 positions in {el:.1f} s "
                      f"(get_range dequant + flash_decode_ref, parallel over heads)"}


# -------------------------------------------------------------------- main --
def _compact(d):
    drop = ("metric", "higher_is_better", "scaling", "vs_baseline", "data")
    return {k: v for k, v in d.items() if k not in drop}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="headline CPU baseline sample (s); each sub-config uses a third")
    ap.add_argument("--workload", choices=["all", "gemv", "gemm_cfg2", "sparse_cfg3", "moe_cfg4",
                                           "kv_cfg5", "midm"], default="all",
                    help="all = the headline GEMV line with every config as a sub-object")
    ap.add_argument("--ep-micro", type=int, default=0,
                    help="MoE micro-batches per step (0: 1)")
    ap.add_argument("--sub-steps", type=int, default=0,
                    help="steps of each sub-config (default: max(--steps, 10), at most 200)")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.gpus != ws and ws > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={ws}", file=sys.stderr)
    if args.impl == "reference":
        res = run_reference(args, ws, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    sub_steps = args.sub_steps or min(max(args.steps, 10), 200)
    cpu_s = 0.0 if args.no_cpu_baseline or rank != 0 or ws != 1 else args.cpu_seconds
    sub_cpu = cpu_s / 3
    res = None
    w = args.workload
    if w in ("all", "gemv"):
        res = run_gemv(args, ws, rank, local, torch, dist, device)
        if cpu_s > 0:
            res["cpu_baseline"] = cpu_baseline(cpu_s)
    if w in ("all", "moe_cfg4"):
        r = run_moe(args, torch, dist, device, ws, rank, local, sub_steps, sub_cpu)
        res = r if res is None else {**res, "moe_cfg4": _compact(r)}
    if ws == 1:
        for name, fn in (("gemm_cfg2", run_gemm), ("sparse_cfg3", run_sparse),
                         ("kv_cfg5", run_kv), ("midm", run_midm)):
            if w == name or (w == "all" and name != "midm"):
                torch.cuda.empty_cache()
                r = fn(args, torch, dist, device, local, sub_steps, sub_cpu)
                res = r if res is None else {**res, name: _compact(r)}
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
