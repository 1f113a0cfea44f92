"""Benchmark of the ternary hot path (one JSON line on stdout from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the metric's "ternary GEMV HBM GB/s"):
dense ternary GEMV, x f32 [1, 2048] ~ N(0,1), W [5632, 2048] ternary with
P(-1)=P(0)=P(+1)=1/3 packed in the reference's 2-bit layout, per-row scales
~ U(0.01, 0.1).  One step = one GEMV y = scale * (W x) on one weight copy.
The steps rotate over R distinct weight copies whose total size exceeds 2x
the 126 MB L2, so every step streams its weights from HBM.  Inputs are made
on the device from a seeded generator (synthetic data; no dataset exists for
this path).

value: algorithmic GB/s over all ranks = steps * ranks * 2,936,832 B / max
over ranks of the device time of the K timed steps (CUDA events on the
launching stream; launches replayed from CUDA graphs).

Multi-GPU: the GEMV does not shard; each rank runs its own replica stream
(weak scaling, no collective on the data path).  Rank 0 prints the line.

--impl reference times the reference's CPU algorithm for the same workload:
the C restatement of ternary_matmul_packed_parallel (src/model/ternary.rs:
471-529) with per-row scales, on all host cores (the reference itself is Rust
and cannot be built on this image; see oracle/).
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
METRIC = "ternary GEMV HBM GB/s"
UNIT = "GB/s"
L2_BYTES = 126 * 1024 * 1024


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        return json.load(open(p))
    except Exception:
        return {}


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


# ------------------------------------------------------------------ ours --
def make_weights(gpu, torch, n_copies, device):
    """n_copies ternary [ROWS, COLS] matrices with row scales, made on the device."""
    weights = []
    g = torch.Generator(device=device)
    for i in range(n_copies):
        g.manual_seed(i)
        codes = torch.randint(0, 3, (ROWS * COLS,), generator=g, device=device, dtype=torch.int32)
        c = codes.view(-1, 16)
        shifts = torch.arange(0, 32, 2, device=device, dtype=torch.int64)
        words = (c.to(torch.int64) << shifts).sum(dim=1)  # 16 codes per u32, LSB first
        words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32).contiguous()
        scales = (torch.rand(ROWS, generator=g, device=device) * 0.09 + 0.01).contiguous()
        import ctypes as C
        h = C.c_void_p()
        ctx = gpu.get_context(device.index)
        from ferrisres_b200._lib import call
        call("ft_weight_from_device_u32", ctx.handle, C.c_void_p(words.data_ptr()), ROWS, COLS,
             C.c_void_p(scales.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream),
             C.byref(h))
        torch.cuda.synchronize()
        weights.append(gpu.DeviceTernaryWeight(h, ROWS, COLS, ctx))
        del codes, words
    return weights


def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist

    from ferrisres_b200 import _lib, gpu

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    group = args.group
    n_copies = max(8, -(-2 * L2_BYTES // (ROWS * COLS // 4)))  # > 2x L2 of weights
    n_copies = -(-n_copies // max(group, 16)) * max(group, 16)
    weights = make_weights(gpu, torch, n_copies, device)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    x = torch.randn(1, COLS, generator=g, device=device)
    ys = [torch.empty(1, ROWS, device=device) for _ in range(n_copies)]
    # one grouped call per G consecutive weight copies, all reading the token x
    calls = [gpu.GroupCall(weights[i:i + group], [x] * group, ys[i:i + group])
             for i in range(0, n_copies, group)]
    singles = [gpu.GroupCall([weights[i]], [x], [ys[i]]) for i in range(n_copies)]

    stream = torch.cuda.Stream(device=device)
    with torch.cuda.stream(stream):  # warm-up; also sizes workspaces before capture
        for i in range(max(args.warmup // group, 3)):
            calls[i % len(calls)]()
        for i in range(3):
            singles[i]()
    stream.synchronize()

    def capture(fns):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for f in fns:
                f()
        return graph

    steps = args.steps
    launches0 = _lib.lib().ft_launch_counter()
    g_full = capture(calls)  # one sweep = n_copies steps
    per_sweep = _lib.lib().ft_launch_counter() - launches0
    full, rem = divmod(steps, n_copies)
    rem_groups, rem_single = divmod(rem, group)
    launches0 = _lib.lib().ft_launch_counter()
    g_rem = capture(calls[:rem_groups] + singles[rem_groups * group:rem_groups * group + rem_single]) \
        if rem else None
    rem_launches = _lib.lib().ft_launch_counter() - launches0
    gpu_launches = full * per_sweep + rem_launches

    def timed(graph_list):
        with torch.cuda.stream(stream):
            graph_list[0][0].replay()  # warm
        stream.synchronize()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for gr, reps in graph_list:
                for _ in range(reps):
                    gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        if ws > 1:
            dist.barrier()
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(local)
    sampler.start()
    plan = [(g_full, full)] + ([(g_rem, 1)] if g_rem is not None else [])
    ms = timed(plan)
    clocks = sampler.stop()
    sec = ms / 1e3
    value = steps * ws * ALGO_BYTES / sec / 1e9

    # smaller launches: 16 GEMVs per launch over the same weights
    calls16 = [gpu.GroupCall(weights[i:i + 16], [x] * 16, ys[i:i + 16])
               for i in range(0, n_copies, 16)]
    g16 = capture(calls16)
    reps16 = max(1, min(full, 20))
    ms16 = timed([(g16, reps16)])
    g16_launch_s = ms16 / 1e3 / (reps16 * len(calls16))
    del g16

    # dependent-chain reference: the same steps as single-GEMV launches
    g_chain = capture(singles)
    chain_reps = max(1, min(full, 20))
    ms_chain = timed([(g_chain, chain_reps)])
    chain_step_s = ms_chain / 1e3 / (chain_reps * n_copies)
    del g_chain

    # end to end through the host-buffer accelerator call (pinned host memory)
    import numpy as np
    acc = gpu.GpuMatmulAccelerator(local)
    xh = torch.empty(COLS, dtype=torch.float32, pin_memory=True)
    xh.copy_(x.view(-1).cpu())
    n_e2e = min(args.steps, 2000)
    t0 = time.perf_counter()
    for i in range(n_e2e):
        acc.gpu_ternary_matmul_vram(weights[i % n_copies], xh.numpy(), 1, COLS, ROWS)
    e2e_sec = time.perf_counter() - t0
    e2e_local = torch.tensor([e2e_sec / n_e2e], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(e2e_local, op=dist.ReduceOp.MAX)
    e2e_value = ws * ALGO_BYTES / float(e2e_local.item()) / 1e9

    peak, peak_kind = load_peaks()
    traffic = load_traffic().get("gemv_cfg0", {}).get("dram_bytes_per_launch")
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": "cfg0 dense ternary GEMV x f32 [1,2048] . W [5632,2048]^T, "
                               "per-row scales", "rows": ROWS, "cols": COLS, "seq": 1,
                   "weight_copies": n_copies,
                   "l2": f"weights rotate over {n_copies} copies "
                         f"({n_copies * ROWS * COLS // 4 / 2**20:.0f} MiB > 2x L2)",
                   "parallelism": f"replicas x{ws}", "graph": "CUDA graph replay",
                   "launch_group": f"{group} GEMVs (shared token x) per launch, e.g. the "
                                   "expert projections of one decode step"},
        "roofline": {"bound": "hbm", "achieved": round(ALGO_BYTES * group / (sec * group / steps) / 1e9, 2),
                     "peak": peak, "unit": "GB/s",
                     "frac": round(ALGO_BYTES * group / (sec * group / steps) / 1e9 / peak, 4),
                     "peak_source": peak_kind, "traffic": traffic,
                     "kernel": "gemv_kernel<1> (activation prep fused)",
                     "algorithmic_bytes_per_launch": ALGO_BYTES * group,
                     "note": f"one launch = {group} GEMVs; achieved = algorithmic bytes per "
                             "launch / per-launch device time (CUDA events over the timed region)"},
        "launch_of_16": {"GBps": round(16 * ALGO_BYTES / g16_launch_s / 1e9, 2),
                         "frac": round(16 * ALGO_BYTES / g16_launch_s / 1e9 / peak, 4),
                         "us_per_launch": round(g16_launch_s * 1e6, 3),
                         "note": "the same GEMVs, 16 per launch"},
        "single_gemv_chain": {"us_per_gemv": round(chain_step_s * 1e6, 3),
                              "GBps": round(ALGO_BYTES / chain_step_s / 1e9, 2),
                              "frac": round(ALGO_BYTES / chain_step_s / 1e9 / peak, 4),
                              "note": "each GEMV its own launch (prep + matmul), back to back "
                                      "in a CUDA graph with programmatic dependent launch"},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": COLS * 4,
                "d2h_bytes_per_step": ROWS * 4, "steps": n_e2e,
                "api": "ft_gpu_ternary_matmul_vram (GpuMatmulAccelerator::gpu_ternary_matmul_vram)"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks,
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    del g_full, g_rem
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ------------------------------------------------------------- CPU side --
CPU_COPIES = 128


def cpu_setup():
    import numpy as np

    from oracle import oracle as fo
    rng = np.random.default_rng(0)
    t = rng.integers(-1, 2, size=ROWS * COLS).astype(np.int8)
    packed = fo.pack_ternary(t)
    rs = rng.uniform(0.01, 0.1, ROWS).astype(np.float32)
    x = rng.standard_normal(COLS).astype(np.float32)
    # the GPU arm's rotation: CPU_COPIES separate copies of the weights (352 MiB),
    # so the timed GEMVs stream them from memory rather than from the last-level cache
    copies = [packed.copy() for _ in range(CPU_COPIES)]
    return fo, copies, rs, x


def cpu_baseline(seconds):
    """Oracle restatement of ternary_matmul_packed_parallel timed on all host cores."""
    fo, copies, rs, x = cpu_setup()
    threads = fo.num_threads(0)
    fo.ternary_matmul_packed_parallel_rows(copies[0], rs, x, ROWS, COLS, threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        fo.ternary_matmul_packed_parallel_rows(copies[n % CPU_COPIES], rs, x, ROWS, COLS, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    return {"value": round(n * ALGO_BYTES / el / 1e9, 3), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{n} GEMVs [5632x2048] in {el:.1f} s (ternary_matmul_packed_parallel, "
                      f"per-row scales, 32 row batches over {threads} threads; weights rotated "
                      f"over {CPU_COPIES} copies, 352 MiB, as in the GPU arm)"}


def run_reference(args, ws, rank):
    if rank != 0:
        return None
    fo, copies, rs, x = cpu_setup()
    threads = fo.num_threads(0)
    for i in range(args.warmup):
        fo.ternary_matmul_packed_parallel_rows(copies[i % CPU_COPIES], rs, x, ROWS, COLS, threads)
    steps = args.steps if args.steps <= 2000 else 2000  # bounded sample
    t0 = time.perf_counter()
    for i in range(steps):
        fo.ternary_matmul_packed_parallel_rows(copies[i % CPU_COPIES], rs, x, ROWS, COLS, threads)
    el = time.perf_counter() - t0
    value = steps * ALGO_BYTES / el / 1e9
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": ws, "steps": steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": "cfg0 dense ternary GEMV x f32 [1,2048] . W [5632,2048]^T, "
                               "per-row scales", "rows": ROWS, "cols": COLS, "seq": 1,
                   "weight_copies": CPU_COPIES},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{steps} GEMVs (requested {args.steps}); C restatement of "
                                   "ternary_matmul_packed_parallel, src/model/ternary.rs:471-529; "
                                   f"weights rotated over {CPU_COPIES} copies (352 MiB), as in "
                                   "the GPU arm"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------- cfg2 GEMM --
G_M, G_K, G_N = 512, 4096, 11008
G_OPS = 2 * G_M * G_K * G_N


def run_gemm(args, ws, rank, local):
    """int8 prefill GEMM (bf16 x -> per-token absmax int8 ->
    exact int32 ternary matmul -> f32), W [11008, 4096] with P(0)=0.5.  One step
    = quantize + matmul; weights rotate over copies totalling > 2x L2."""
    import torch

    from ferrisres_b200 import _lib, gpu

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    n_copies = max(3, -(-2 * L2_BYTES // (G_N * G_K // 4)))
    weights = []
    g = torch.Generator(device=device)
    import ctypes as C
    from ferrisres_b200._lib import call
    ctx = gpu.get_context(local)
    for i in range(n_copies):
        g.manual_seed(100 + i)
        u = torch.rand(G_N * G_K, generator=g, device=device)
        codes = torch.where(u < 0.25, 0, torch.where(u < 0.75, 1, 2)).to(torch.int64)
        words = (codes.view(-1, 16) << torch.arange(0, 32, 2, device=device)).sum(dim=1)
        words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32).contiguous()
        scales = (torch.rand(G_N, generator=g, device=device) * 0.09 + 0.01).contiguous()
        h = C.c_void_p()
        call("ft_weight_from_device_u32", ctx.handle, C.c_void_p(words.data_ptr()), G_N, G_K,
             C.c_void_p(scales.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream),
             C.byref(h))
        torch.cuda.synchronize()
        weights.append(gpu.DeviceTernaryWeight(h, G_N, G_K, ctx))
        del u, codes, words
    g.manual_seed(7)
    xb = torch.randn(G_M, G_K, generator=g, device=device).to(torch.bfloat16)
    y = torch.empty(G_M, G_N, device=device)
    stream = torch.cuda.Stream(device=device)

    def step(i):
        q, sx = gpu.quantize_absmax_i8(xb)
        weights[i % n_copies].matmul_i8(q, sx, out=y)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
    stream.synchronize()
    launches0 = _lib.lib().ft_launch_counter()
    with torch.cuda.stream(stream):
        step(0)
    per_step = _lib.lib().ft_launch_counter() - launches0
    stream.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    sec = e0.elapsed_time(e1) / 1e3
    tops = args.steps * G_OPS / sec / 1e12
    bf16_peak = None
    try:
        bf16_peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
    except Exception:
        pass
    peak = 2 * (bf16_peak or 1590.0)
    return {
        "metric": "ternary int8 prefill GEMM TOPS", "value": round(tops, 2), "unit": "TOPS",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded, generated on device)",
        "config": {"workload": "cfg2 prefill GEMM M=512 K=4096 N=11008, bf16 x -> absmax int8",
                   "weight_copies": n_copies, "l2": "weights rotate over copies > 2x L2"},
        "roofline": {"bound": "tensor", "achieved": round(tops, 2), "peak": round(peak, 1),
                     "unit": "TOP/s", "frac": round(tops / peak, 4),
                     "peak_source": "2 x measured bf16 dense (int8 dense rate is twice bf16 on B200)"
                                    if bf16_peak else "2 x fallback bf16",
                     "traffic": load_traffic().get("gemm_cfg2", {}).get("dram_bytes_per_launch"),
                     "kernel": "tq_grouped_kernel<128, 0> (+ prep_b_kernel, quantize_i8_kernel)",
                     "note": "achieved = the whole step's int ops (quantize + prep + matmul) / "
                             "step time"},
        "gpu_launches": int(per_step * args.steps),
        "clocks": clocks,
    }


# ------------------------------------------------------------ cfg3 2:4 ---
S_N, S_K = 14336, 4096


def run_sparse(args, ws, rank, local):
    """2:4 sparse ternary matmul, K=4096, N=14336, fp32 x,
    at M=1 (bandwidth-bound decode GEMV kernel, grouped launches of --group)
    and M=64 (tensor-core engine).
    Weights enter in the reference SparseTernaryMatrix layout and are stored
    at 1.25 bits/weight; copies rotate beyond 2x L2."""
    import numpy as np
    import torch

    from ferrisres_b200 import _lib, gpu

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dev_bytes = (S_N // 128) * (S_K // 128) * 2560
    algo = dev_bytes + S_N * 4 + S_K * 4 + S_N * 4  # weights + scales + x + y per GEMV
    group = min(args.group, 64)
    n_copies = -(-max(4, -(-2 * L2_BYTES // dev_bytes)) // group) * group
    rng = np.random.default_rng(0)
    ng = S_N * S_K // 4
    weights = []
    for i in range(n_copies):
        if i < 8:  # 8 distinct matrices, uploaded as separate copies beyond that
            lo = rng.integers(0, 6, size=(ng + 1) // 2, dtype=np.uint8)
            hi = rng.integers(0, 6, size=(ng + 1) // 2, dtype=np.uint8)
            pat = (lo | (hi << 4)).astype(np.uint8)
            sg = rng.integers(0, 256, size=(ng + 3) // 4, dtype=np.uint8)
            rs = rng.uniform(0.01, 0.1, S_N).astype(np.float32)
        weights.append(gpu.DeviceTernaryWeight.from_sparse_host(pat, sg, S_N, S_K, rs, local))
    assert weights[0].device_bytes() == dev_bytes + S_N * 4
    x1 = torch.randn(1, S_K, device=device)
    x64 = torch.randn(64, S_K, device=device)
    ys = [torch.empty(1, S_N, device=device) for _ in range(n_copies)]
    y64 = torch.empty(64, S_N, device=device)
    calls = [gpu.GroupCall(weights[i:i + group], [x1] * group, ys[i:i + group])
             for i in range(0, n_copies, group)]
    stream = torch.cuda.Stream(device=device)
    with torch.cuda.stream(stream):
        for c in calls:
            c()
        weights[0].matmul_f32(x64, out=y64)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for c in calls:
            c()
    reps = max(1, args.steps // n_copies)
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    sec = e0.elapsed_time(e1) / 1e3
    gbps = reps * n_copies * algo / sec / 1e9
    # M = 64 (one matmul per step, weights rotating)
    m64_steps = max(4, min(args.steps, 200))
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(m64_steps):
            weights[i % n_copies].matmul_f32(x64, out=y64)
        e1.record(stream)
    torch.cuda.synchronize()
    sec64 = e0.elapsed_time(e1) / 1e3 / m64_steps
    peak, peak_kind = load_peaks()
    return {
        "metric": "2:4 sparse ternary GEMV HBM GB/s", "value": round(gbps, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": reps * n_copies, "warmup": n_copies,
        "ms_per_step": sec * 1e3 / (reps * n_copies), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded 2:4 patterns and signs)",
        "config": {"workload": "cfg3 2:4 sparse K=4096 N=14336, M=1 (grouped) and M=64",
                   "device_bytes_per_weight": dev_bytes, "bits_per_weight": 1.25,
                   "launch_group": group, "weight_copies": n_copies},
        "roofline": {"bound": "hbm", "achieved": round(gbps, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(gbps / peak, 4), "peak_source": peak_kind,
                     "algorithmic_bytes_per_gemv": algo,
                     "traffic": load_traffic().get("sparse_cfg3", {}).get("dram_bytes_per_launch"),
                     "traffic_launch": "64 GEMVs", "kernel": "gemv_kernel<1,64,true>"},
        "m64": {"ms": round(sec64 * 1e3, 4), "TOPS_nonzero": round(2 * 64 * S_N * S_K / 2 / sec64 / 1e12, 2),
                "GBps_weights": round(dev_bytes / sec64 / 1e9, 1)},
        "gpu_launches": int(reps * len(calls)),  # one decode-GEMV launch per grouped call
        "clocks": clocks,
    }


# ------------------------------------------------------------- cfg4 MoE ---
M_E, M_H, M_F, M_T, M_K = 64, 2048, 1408, 4096, 2
M_OPS = M_T * M_K * (3 * 2 * M_H * M_F) + 2 * M_T * M_E * M_H


def _rand_packed(rng, rows, cols):
    """Reference pack_ternary bytes of a matrix with P(-1)=P(0)=P(+1)=1/3."""
    c = rng.integers(0, 3, size=(rows * cols // 4, 4), dtype=np.uint8)
    return (c[:, 0] | (c[:, 1] << 2) | (c[:, 2] << 4) | (c[:, 3] << 6)).astype(np.uint8)


def run_moe(args, ws, rank, local):
    """ternary MoE FFN layer, 64 experts, H=2048, F=1408,
    SwiGLU, top-2, 4096 bf16 tokens; expert-parallel over the ranks (rank r
    holds experts [r*64/N, (r+1)*64/N) and routes 4096/N tokens).  One step = one
    layer forward over the global batch.  value = 4096 tokens / max-over-ranks
    device time (strong scaling: the layer and batch are fixed)."""
    import datetime

    import torch
    import torch.distributed as dist

    from ferrisres_b200 import moe, moe_ep

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    rng = np.random.default_rng(4)
    router = (rng.standard_normal(M_E * M_H) * 0.02).astype(np.float32)
    router = torch.from_numpy(router).to(torch.bfloat16).float().numpy()  # bf16 router weights
    per = M_E // ws
    mine = range(rank * per, (rank + 1) * per)
    g, u, d, gs, us, ds = [], [], [], [], [], []
    for e in range(M_E):
        wrng = np.random.default_rng(1000 + e)
        if e in mine:
            g.append(_rand_packed(wrng, M_F, M_H)); u.append(_rand_packed(wrng, M_F, M_H))
            d.append(_rand_packed(wrng, M_H, M_F))
            gs.append(wrng.uniform(0.01, 0.1, M_F).astype(np.float32))
            us.append(wrng.uniform(0.01, 0.1, M_F).astype(np.float32))
            ds.append(wrng.uniform(0.01, 0.1, M_H).astype(np.float32))
        else:
            for lst in (g, u, d, gs, us, ds):
                lst.append(None)
    layer = moe.TernaryMoELayer(router, g, gs, u, us, d, ds, M_H, M_F, M_K, device=local)
    be = moe_ep.GpuMoEBackend(layer)
    gx = torch.Generator(device=device).manual_seed(99)
    x = torch.randn(M_T, M_H, generator=gx, device=device).to(torch.bfloat16)
    shard = x.chunk(ws)[rank].contiguous()
    stream = torch.cuda.Stream(device=device)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            moe_ep.ep_forward(shard, be, M_E, rank, ws)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            moe_ep.ep_forward(shard, be, M_E, rank, ws)
        e1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    sec = float(t.item()) / args.steps
    res = {
        "metric": "MoE-layer tokens/s", "value": round(M_T / sec, 1), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded ternary experts, bf16 router and tokens)",
        "config": {"workload": "cfg4 ternary MoE FFN: 64 experts, H=2048, F=1408, SwiGLU, top-2, "
                               "4096 tokens", "parallelism": f"ep{ws}",
                   "experts_per_gpu": per, "tokens_per_gpu": M_T // ws},
        "algorithmic_TOPS": round(M_OPS / sec / 1e12, 2),
        "clocks": clocks,
    }
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


# ---------------------------------------------------------- cfg5 3-bit KV --
KV_B, KV_HQ, KV_HKV, KV_D, KV_S = 32, 32, 8, 128, 32768
KV_CACHE_BYTES = KV_B * KV_HKV * KV_S * (48 + 48 + 8 + 8)  # codes + (min, max), K and V
KV_IO_BYTES = 2 * KV_B * KV_HQ * KV_D * 4                  # q in, out
KV_ALGO_BYTES = KV_CACHE_BYTES + KV_IO_BYTES


def run_kv(args, ws, rank, local):
    """TurboQuant 3-bit KV flash decode, B=32, Hq=32, Hkv=8,
    d=128, context 32768 (reference scheme: per-vector min/max, 3-bit codes).
    One step = append one position per sequence (bf16 K, V) + evict the oldest
    (the context stays at 32768) + flash decode over the cache.  value = the
    step's algorithmic bytes (cache read + q/out) / device time, over all ranks
    (replicas: each rank decodes its own batch)."""
    import torch
    import torch.distributed as dist

    from ferrisres_b200 import _lib, kv

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    cache = kv.Kv3Cache(KV_B, KV_HKV, KV_S + 64, device=local)
    gen = torch.Generator(device=device).manual_seed(5 + rank)
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

    def step():
        cache.append(k1, v1, stream=stream)
        cache.evict_front(1)
        cache.flash_decode(q, out=out, stream=stream)

    for _ in range(max(args.warmup, 3)):
        step()
    stream.synchronize()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=device, dtype=torch.float64)
        if ws > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    launches0 = _lib.lib().ft_launch_counter()
    sampler = ClockSampler(local)
    sampler.start()
    sec = timed(step, args.steps)
    clocks = sampler.stop()
    gpu_launches = _lib.lib().ft_launch_counter() - launches0
    # the dominant kernel alone (decode + split combine), for the roofline
    n_dec = max(5, min(args.steps, 50))
    dec_sec = timed(lambda: cache.flash_decode(q, out=out, stream=stream), n_dec) / n_dec
    step_s = sec / args.steps
    value = ws * KV_ALGO_BYTES / step_s / 1e9

    # end to end through the public API with host buffers: q and the new K/V
    # from pinned host memory, the output read back every step
    qh = torch.empty_like(q, device="cpu").pin_memory()
    qh.copy_(q.cpu())
    kh = torch.empty_like(k1, device="cpu").pin_memory()
    kh.copy_(k1.cpu())
    oh = torch.empty_like(out, device="cpu").pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k1), torch.empty_like(v1)
    n_e2e = max(3, min(args.steps, 50))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(n_e2e):
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(kh, non_blocking=True)
            cache.append(kd, vd, stream=stream)
            cache.evict_front(1)
            cache.flash_decode(qd, out=out, stream=stream)
            oh.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3 / n_e2e], device=device, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = ws * KV_ALGO_BYTES / float(t.item()) / 1e9
    cache.ctx.check()

    peak, peak_kind = load_peaks()
    traffic = load_traffic().get("kv_cfg5", {}).get("dram_bytes_per_launch")
    dec_gbs = KV_ALGO_BYTES / dec_sec / 1e9
    res = {
        "metric": "3-bit KV flash-decode HBM GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 codes / f32",
        "data": "synthetic (K, V ~ N(0,1) bf16 quantised to 3 bits; q ~ N(0,1))",
        "config": {"workload": "cfg5 3-bit KV flash decode: B=32, Hq=32, Hkv=8, d=128, ctx 32768, "
                               "reference TurboQuantKVCache scheme (min/max per 128-vector)",
                   "step": "append 1 position + evict oldest + decode",
                   "l2": f"cache {KV_CACHE_BYTES / 2**20:.0f} MiB > L2",
                   "parallelism": f"replicas x{ws}",
                   "decode_tokens_per_s": round(ws * KV_B / step_s, 1)},
        "roofline": {"bound": "hbm", "achieved": round(dec_gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(dec_gbs / peak, 4), "peak_source": peak_kind,
                     "traffic": traffic, "kernel": "kv3_decode_kernel (+ kv3_combine_kernel)",
                     "algorithmic_bytes_per_launch": KV_ALGO_BYTES,
                     "note": "112 B per (sequence, position, kv head) + q/out; decode launch "
                             "timed alone with CUDA events"},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": q.numel() * 4 + 2 * k1.numel() * 2,
                "d2h_bytes_per_step": out.numel() * 4, "steps": n_e2e,
                "api": "Kv3Cache.append + flash_decode (ft_kv3_append, ft_flash_decode_3bit)"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks,
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = kv_cpu_baseline(args.cpu_seconds)
    cache.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--group", type=int, default=64, help="GEMVs per launch (1..64)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--workload", choices=["gemv", "gemm_cfg2", "sparse_cfg3", "moe_cfg4", "kv_cfg5"],
                    default="gemv",
                    help="gemv = the headline cfg0 line; gemm_cfg2 = the int8 prefill GEMM")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.gpus != ws and ws > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={ws}", file=sys.stderr)
    if args.workload == "gemm_cfg2" and args.impl == "ours":
        res = run_gemm(args, ws, rank, local)
    elif args.workload == "sparse_cfg3" and args.impl == "ours":
        res = run_sparse(args, ws, rank, local)
    elif args.workload == "moe_cfg4" and args.impl == "ours":
        res = run_moe(args, ws, rank, local)
    elif args.workload == "kv_cfg5" and args.impl == "ours":
        res = run_kv(args, ws, rank, local)
    elif args.impl == "reference":
        res = run_reference(args, ws, rank)
    else:
        res = run_ours(args, ws, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
