#!/usr/bin/env python
"""Headline benchmark: exact flat k-NN, queries/sec at N=10M, d=768, k=10 (squared L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one batch of Q=10,000 queries searched against the whole database. The database
(N = 10,000,000 x 768 fp32, TestRNG N(0,1) seed 0, stream = row) is row-sharded across the ranks
(N/world rows each, global ids = shard base + local row); queries (seed 1, streams offset 2^31)
go to every rank. Each rank searches its shard (tensor-core bf16 filter + exact fp64 rerank, one
stream), the per-rank top-k lists are all-gathered over NCCL and merged on the device.

value   = whole-job queries/s with queries resident in HBM (device time, max over ranks)
e2e     = queries/s through the public host-buffer entry point: pinned host queries copied in
          and results copied out inside the timed region
roofline: the tensor-core filter kernel, 2*Q*N_local*d FLOP per launch over its CUDA-event time,
          against MEASURED_PEAKS.json's sustained bf16 GEMM figure
cpu_baseline: the CPU oracle (a C++ restatement of the reference's CPUTopK / vDSP path, fp32,
          all host threads) timed on a bounded sample on rank 0 at N=1

--impl reference runs only that CPU restatement (the reference itself is Swift + Metal and
cannot run on Linux), on rank 0, and prints the same JSON line with "impl": "reference".
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "queries/sec at N=10M d=768 k=10 (1/2/4/8 B200); % tensor-pipe / HBM roofline"
QUERY_ROW0 = 1 << 31


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n", type=int, default=10_000_000)
    p.add_argument("--dim", type=int, default=768)
    p.add_argument("--nq", type=int, default=10_000)
    p.add_argument("--k", type=int, default=10)
    p.add_argument("--precision", choices=["bf16", "tf32", "fp32"], default="bf16")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-rows", type=int, default=1_000_000, help="database rows of the CPU sample")
    p.add_argument("--no-clocks", action="store_true")
    p.add_argument("--config", choices=["headline"] + sorted(CONFIGS) + ["ivf"], default="headline",
                   help="headline (the default bench line), one of the other BASELINE configurations, or ivf "
                        "(the IVF search, not a BASELINE configuration)")
    p.add_argument("--nlist", type=int, default=1024, help="ivf: inverted lists")
    p.add_argument("--nprobe", type=int, default=32, help="ivf: lists probed per query")
    p.add_argument("--kmeans-iters", type=int, default=20, help="ivf: k-means iteration limit")
    p.add_argument("--kmeans-tol", type=float, default=1e-3, help="ivf: k-means movement threshold")
    a = p.parse_args()
    if a.config == "ivf":
        for key, v in (("n", 1_000_000), ("dim", 128), ("nq", 10_000), ("k", 10)):
            if getattr(a, key) == p.get_default(key):
                setattr(a, key, v)
    elif a.config != "headline":
        # the other configurations carry their own sizes unless given explicitly
        c = CONFIGS[a.config]
        for key in ("n", "dim", "nq", "k"):
            if getattr(a, key) == p.get_default(key):
                setattr(a, key, c[key])
    return a


# Other BASELINE configurations (seeded synthetic stand-ins, generated on the device). Mixture rows:
# centroid c (TestRNG, seed ^ const, stream c) + sigma * N(0,1) (seed, stream = row), optionally
# unit-normalised; queries come from the same mixture on streams offset by 2^31.
CONFIGS = {
    "c2": dict(desc="flat cosine k-NN, mixture of 1,024 centroids sigma 0.3, L2-normalised",
               n=1_000_000, dim=1536, nq=10_000, k=100, kind="float", metric="COSINE", rows="f32",
               mixture=(1024, 0.3, True), rerank=0),
    "c3": dict(desc="sharded flat max-inner-product k-NN, bf16 rows, mixture of 4,096 centroids sigma 0.25, "
                    "normalised; exact rerank of the top 4k", n=50_000_000, dim=768, nq=4096, k=10, kind="float",
               metric="IP", rows="bf16", mixture=(4096, 0.25, True), rerank=4),
    "c4": dict(desc="int8 scalar-quantized L2 k-NN (per-dimension min/max over the database), mixture of 2,048 "
                    "centroids sigma 0.3; int32 L2 on codes, exact fp32-row rerank of the top 1,000",
               n=20_000_000, dim=768, nq=8192, k=100, kind="int8", mixture=(2048, 0.3, False), candidates=1000),
    "c5": dict(desc="Hamming k-NN over sign bits of N(0,1) d=1024 (database seed 2, queries seed 3)",
               n=200_000_000, dim=1024, nq=1024, k=100, kind="binary"),
    "c5q1": dict(desc="Hamming k-NN, single query (latency), sign bits of N(0,1) d=1024 (seeds 2 / 3)",
                 n=200_000_000, dim=1024, nq=1, k=100, kind="binary"),
}


def workload(a):
    return {
        "workload": f"flat exact squared-L2 k-NN: database N={a.n:,} x d={a.dim} fp32 (TestRNG N(0,1) seed 0), "
                    f"Q={a.nq:,} queries (seed 1), k={a.k}",
        "N": a.n, "d": a.dim, "Q": a.nq, "k": a.k, "metric": "L2SQ",
        "global_batch": a.nq,
        "l2_policy": "inputs larger than L2 (database operand >> 126 MB), no flush",
    }


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ------------------------------------------------------------------------------------------ CPU baseline
def cpu_baseline(a, steps: int = 1, warmup: int = 0):
    """Oracle port on host cores, bounded sample: Qs queries x the first cpu_rows database rows,
    scaled to full N (per-query cost is linear in N)."""
    from oracle import oracle
    threads = os.cpu_count() or 1
    rows = min(a.cpu_rows, a.n)
    qs = max(64, 8 * threads)
    x = oracle.gen_gaussian(rows, a.dim, 0, threads=threads)
    q = oracle.gen_gaussian(qs, a.dim, 1, row0=QUERY_ROW0, threads=threads)
    for _ in range(warmup):
        oracle.knn(q, x, a.k, truth=False, threads=threads)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle.knn(q, x, a.k, truth=False, threads=threads)
        times.append(time.perf_counter() - t0)
    t = float(np.mean(times))
    qps = qs / t * rows / a.n
    return {
        "value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
        "sample": f"{qs} queries x first {rows:,} of {a.n:,} rows (fp32, all host threads), "
                  f"{t:.3f} s per sample; QPS scaled by {rows:,}/{a.n:,} (cost linear in N)",
    }, t


def run_reference(a):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    base, t = cpu_baseline(a, steps=a.steps, warmup=min(a.warmup, 1))
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "queries/s", "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (TestRNG restatement)",
        "config": workload(a), "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "VectorAccelerate is Swift + Metal + Accelerate (macOS only); its CPU search path "
                "(CPUTopK.swift / vDSP) is timed as the C++ restatement in oracle/ on this host's cores",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str, enabled: bool = True):
        self.proc = None
        self.path = os.path.join(ROOT, "_work", f"clocks_{os.getpid()}.csv")
        if not enabled:
            return
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", gpus, "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.remove(self.path)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}, "fallback"


def profiled_traffic():
    """DRAM bytes per filter launch from the committed ncu summary (scaled per unit), or None."""
    path = os.path.join(ROOT, "profiles", "tc_filter_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return None


# ------------------------------------------------------------------------------------------ ours
def run_ours(a):
    import torch
    import torch.distributed as dist

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    # One explicit stream shared by the library, torch copies and NCCL (the legacy default
    # stream would make the library create its own, unordered with the timing events).
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx = va.GPUContext(va.Metal4Configuration(device=local, stream=stream.cuda_stream))
    prec = {"bf16": va.PREC_BF16, "tf32": va.PREC_TF32, "fp32": va.PREC_FP32}[a.precision]

    from vectoraccelerate_b200.sharded import ShardedSearch, device_merge, shard_bounds

    # ---- database shard, generated on the device, built into a resident va_database
    row0, n_local = shard_bounds(a.n, world, rank)
    gen = torch.empty((n_local, a.dim), dtype=torch.float32, device="cuda")
    _ffi.call("va_gen_gaussian", ctx.handle, gen.data_ptr(), n_local, a.dim, 0, row0)
    db = va.Database(ctx, None, device_ptr=gen.data_ptr(), n=n_local, dim=a.dim, id_base=row0)
    ctx.synchronize()
    del gen
    torch.cuda.empty_cache()

    # ---- queries: device copy for `value`, pinned host copy for `e2e`
    dq = torch.empty((a.nq, a.dim), dtype=torch.float32, device="cuda")
    _ffi.call("va_gen_gaussian", ctx.handle, dq.data_ptr(), a.nq, a.dim, 1, QUERY_ROW0)
    ctx.synchronize()
    hq = dq.cpu().pin_memory()
    k = a.k
    lv = torch.empty((a.nq, k), dtype=torch.float32, device="cuda")
    li = torch.empty((a.nq, k), dtype=torch.int32, device="cuda")
    hv = torch.empty((a.nq, k), dtype=torch.float32).pin_memory()
    hi = torch.empty((a.nq, k), dtype=torch.int32).pin_memory()
    launches_per_step = 3 + (1 if world > 1 else 0)  # query operand, filter, merge+rerank (+ shard merge)
    if prec == va.PREC_FP32:
        launches_per_step = None
    qptr = [dq.data_ptr()]

    def local_search(nq, kk):
        _ffi.call("va_knn_search", ctx.handle, db.handle, qptr[0], nq, kk, va.METRIC_L2SQ, prec, 0,
                  lv.data_ptr(), li.data_ptr())
        return lv, li

    sharded = ShardedSearch(world, local_search, device_merge(ctx, world, a.nq, k))
    final = [lv, li]

    def step_device(queries_ptr):
        qptr[0] = queries_ptr
        final[0], final[1] = sharded.search(a.nq, k)

    def step_e2e():
        if world == 1:
            _ffi.call("va_knn_search_host", ctx.handle, db.handle, ctypes.c_void_p(hq.data_ptr()), a.nq, k,
                      va.METRIC_L2SQ, prec, 0, ctypes.c_void_p(hv.data_ptr()), ctypes.c_void_p(hi.data_ptr()))
        else:
            dq.copy_(hq, non_blocking=True)
            step_device(dq.data_ptr())
            hv.copy_(final[0], non_blocking=True)
            hi.copy_(final[1], non_blocking=True)

    def barrier_sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up, plus a sanity check of the result shape (parity itself is tests/' job)
    for _ in range(max(3, a.warmup)):
        step_device(dq.data_ptr())
    barrier_sync()
    ids0 = final[1].cpu().numpy().view(np.uint32)
    vals0 = final[0].cpu().numpy()
    assert (ids0 < a.n).all() and np.all(np.diff(vals0, axis=1) >= 0), "search returned invalid results"

    # ---- device-resident timing
    clocks = ClockSampler(",".join(str(i) for i in range(world)) if rank == 0 else "0",
                          enabled=(rank == 0 and not a.no_clocks))
    _ffi.call("va_profile_start", ctx.handle, a.steps)
    barrier_sync()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.steps):
        step_device(dq.data_ptr())
    e1.record(stream)
    barrier_sync()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    kms = ctypes.c_float()
    kcalls = ctypes.c_int()
    _ffi.call("va_profile_stop", ctx.handle, ctypes.byref(kms), ctypes.byref(kcalls))
    kernel_ms = max_over_ranks(kms.value / max(1, kcalls.value)) if kcalls.value else None

    # ---- end-to-end timing through the host-buffer path
    for _ in range(a.warmup):
        step_e2e()
    barrier_sync()
    e0.record(stream)
    for _ in range(a.steps):
        step_e2e()
    e1.record(stream)
    barrier_sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    if world == 1:
        # va_knn_search_host runs on the context stream and waits; bracket with wall time too
        t0 = time.perf_counter()
        for _ in range(a.steps):
            step_e2e()
        e2e_ms = max(e2e_ms, (time.perf_counter() - t0) * 1e3 / a.steps)

    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    peaks, peak_src = measured_peaks()
    flops = 2.0 * a.nq * n_local * a.dim
    roof = None
    if kernel_ms:
        peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
        if a.precision == "tf32":
            peak = peak / 2.0
        achieved = flops / (kernel_ms * 1e-3) / 1e12
        tr = profiled_traffic()
        traffic = None
        if tr and tr.get("precision") == a.precision:
            traffic = tr["bytes_per_row"] * n_local * (a.nq / tr.get("queries", a.nq))
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": traffic, "kernel": "k_tc_filter", "kernel_ms": kernel_ms,
                "peak_source": f"{peak_src} bf16 sustained" + (" / 2 for tf32" if a.precision == "tf32" else ""),
                "flop_per_launch": flops}
    line = {
        "metric": METRIC, "value": a.nq / (ms * 1e-3), "unit": "queries/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": f"{a.precision} filter + f64 exact rerank",
        "data": "synthetic: TestRNG restatement, N(0,1) database seed 0, queries seed 1 (streams offset 2^31)",
        "config": dict(workload(a), parallelism=f"row-shard x{world}, NCCL allgather + device merge",
                       precision=a.precision),
        "e2e": {"value": a.nq / (e2e_ms * 1e-3), "unit": "queries/s",
                "h2d_bytes_per_step": world * a.nq * a.dim * 4, "d2h_bytes_per_step": world * a.nq * k * 8},
        "gpu_launches": launches_per_step * a.steps if launches_per_step else None,
        "roofline": roof,
        "clocks": clk,
    }
    if world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"], _ = cpu_baseline(a)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------------ other configs
def auto_precision(k: int, rerank: int, f32_rows: bool = True) -> str:
    """The filter precision va_knn_search picks under PREC_AUTO: bf16 when the candidate pool
    (rerank * k, else k + max(k/4, 22), rounded up to 32/64/128 when it fits) holds >= 3k, and,
    without a caller's factor, over fp32 rows (the pool then widens to 3k)."""
    want = rerank * k if rerank else k + max(k // 4, 22)
    pool = next((p for p in (32, 64, 128) if want <= p), want)
    if pool < 3 * k and rerank == 0 and f32_rows and 3 * k <= 4096:
        return "bf16"
    return "bf16" if pool >= 3 * k else "tf32"


def run_config(a):
    """One of the other BASELINE configurations on this rank's row shard (N/world rows, global
    ids = shard base + row), all-gather + device merge for world > 1, as the headline."""
    import torch
    import torch.distributed as dist

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi
    from vectoraccelerate_b200.sharded import ShardedSearch, device_merge, shard_bounds

    c = CONFIGS[a.config]
    kind = c["kind"]
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx = va.GPUContext(va.Metal4Configuration(device=local, stream=stream.cuda_stream))
    n_total = a.n
    note = None
    row0, n_local = shard_bounds(n_total, world, rank)
    dim, nq, k = a.dim, a.nq, a.k
    chunk = max(1, (4 << 30) // (4 * dim))  # fp32 generation chunks of <= 4 GiB

    def gen_f32(dst_ptr, rows, seed, r0):
        if c.get("mixture"):
            nc, sigma, norm = c["mixture"]
            _ffi.call("va_gen_mixture", ctx.handle, dst_ptr, rows, dim, seed, r0, nc, sigma, int(norm))
        else:
            _ffi.call("va_gen_gaussian", ctx.handle, dst_ptr, rows, dim, seed, r0)

    db_seed, q_seed, q_row0 = (2, 3, 0) if kind == "binary" else (0, 0, QUERY_ROW0)
    # ---- database shard
    if kind == "float" and c["rows"] == "bf16":
        rows = torch.empty((n_local, dim), dtype=torch.int16, device="cuda")
        tmp = torch.empty((min(chunk, n_local), dim), dtype=torch.float32, device="cuda")
        for r in range(0, n_local, chunk):
            m = min(chunk, n_local - r)
            gen_f32(tmp.data_ptr(), m, db_seed, row0 + r)
            _ffi.call("va_f32_to_bf16", ctx.handle, tmp.data_ptr(), m * dim, rows[r:r + m].data_ptr())
        ctx.synchronize()
        del tmp
        torch.cuda.empty_cache()
        db = va.Database(ctx, None, dtype=va.DTYPE_BF16, device_ptr=rows.data_ptr(), n=n_local, dim=dim,
                         id_base=row0)
    elif kind in ("float", "int8"):
        rows = torch.empty((n_local, dim), dtype=torch.float32, device="cuda")
        for r in range(0, n_local, chunk):
            gen_f32(rows[r:].data_ptr(), min(chunk, n_local - r), db_seed, row0 + r)
        ctx.synchronize()
        if kind == "float":
            db = va.Database(ctx, None, device_ptr=rows.data_ptr(), n=n_local, dim=dim, id_base=row0)
        else:
            # per-dimension range over the WHOLE database: local min / max, then MIN / MAX all-reduce
            mn = torch.empty(dim, dtype=torch.float32, device="cuda")
            mx = torch.empty(dim, dtype=torch.float32, device="cuda")
            _ffi.call("va_sq_perdim_minmax", ctx.handle, rows.data_ptr(), n_local, dim, mn.data_ptr(), mx.data_ptr())
            torch.cuda.synchronize()
            if world > 1:
                dist.all_reduce(mn, op=dist.ReduceOp.MIN)
                dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            db = va.Int8Database(ctx, None, id_base=row0, mins=mn.cpu().numpy(), maxs=mx.cpu().numpy(),
                                 device_ptr=rows.data_ptr(), n=n_local, dim=dim)
    else:
        words = dim // 32
        rows = torch.empty((n_local, words), dtype=torch.int32, device="cuda")
        tmp = torch.empty((min(chunk, n_local), dim), dtype=torch.float32, device="cuda")
        for r in range(0, n_local, chunk):
            m = min(chunk, n_local - r)
            gen_f32(tmp.data_ptr(), m, db_seed, row0 + r)
            _ffi.call("va_binary_quantize", ctx.handle, tmp.data_ptr(), m, dim, 0.0, rows[r:r + m].data_ptr())
        ctx.synchronize()
        del tmp
        db = va.BinaryDatabase.from_device(ctx, rows.data_ptr(), n_local, dim, id_base=row0)
    ctx.synchronize()
    del rows
    torch.cuda.empty_cache()

    # ---- queries (device copy for `value`, pinned host copy for `e2e`)
    if kind == "binary":
        qf = torch.empty((nq, dim), dtype=torch.float32, device="cuda")
        gen_f32(qf.data_ptr(), nq, q_seed, q_row0)
        dq = torch.empty((nq, dim // 32), dtype=torch.int32, device="cuda")
        _ffi.call("va_binary_quantize", ctx.handle, qf.data_ptr(), nq, dim, 0.0, dq.data_ptr())
        del qf
    else:
        dq = torch.empty((nq, dim), dtype=torch.float32, device="cuda")
        gen_f32(dq.data_ptr(), nq, q_seed, q_row0)
    ctx.synchronize()
    hq = dq.cpu().pin_memory()
    lv = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    li = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    hv = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    hi = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    metric = {"COSINE": va.METRIC_COSINE, "IP": va.METRIC_IP}.get(c.get("metric"), va.METRIC_L2SQ)
    mode = 1 if metric == va.METRIC_IP and kind == "float" else 0

    def local_search(nq_, kk):
        if kind == "float":
            _ffi.call("va_knn_search", ctx.handle, db.handle, dq.data_ptr(), nq_, kk, metric, va.PREC_AUTO,
                      c["rerank"], lv.data_ptr(), li.data_ptr())
        elif kind == "int8":
            _ffi.call("va_int8_knn_search", ctx.handle, db.handle, dq.data_ptr(), nq_, kk, c["candidates"],
                      lv.data_ptr(), li.data_ptr())
        else:
            # uint32 distances are written as their bit patterns into the float list; those order
            # like the integers, so the float merge applies unchanged
            _ffi.call("va_hamming_knn_db", ctx.handle, db.handle, dq.data_ptr(), nq_, kk, lv.data_ptr(),
                      li.data_ptr())
        return lv, li

    sharded = ShardedSearch(world, local_search, device_merge(ctx, world, nq, k, mode=mode))
    final = [lv, li]

    def step():
        final[0], final[1] = sharded.search(nq, k)

    def step_e2e():
        dq.copy_(hq, non_blocking=True)
        step()
        hv.copy_(final[0], non_blocking=True)
        hi.copy_(final[1], non_blocking=True)

    def barrier_sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, a.warmup)):
        step()
    barrier_sync()
    ids0 = final[1].cpu().numpy().view(np.uint32)
    assert (ids0 < n_total).all(), "search returned invalid ids"

    clocks = ClockSampler(",".join(str(i) for i in range(world)) if rank == 0 else "0",
                          enabled=(rank == 0 and not a.no_clocks))
    _ffi.call("va_profile_start", ctx.handle, a.steps)
    barrier_sync()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    for e0, e1 in evs:
        e0.record(stream)
        step()
        e1.record(stream)
    barrier_sync()
    clk = clocks.stop()
    per = sorted(e0.elapsed_time(e1) for e0, e1 in evs)
    ms = max_over_ranks(float(np.mean(per)))
    p50 = max_over_ranks(per[len(per) // 2])
    p99 = max_over_ranks(per[min(len(per) - 1, int(round(0.99 * (len(per) - 1))))])
    kms, kcalls = ctypes.c_float(), ctypes.c_int()
    _ffi.call("va_profile_stop", ctx.handle, ctypes.byref(kms), ctypes.byref(kcalls))
    kernel_ms = max_over_ranks(kms.value / max(1, kcalls.value)) if kcalls.value else None

    for _ in range(a.warmup):
        step_e2e()
    barrier_sync()
    e0, e1 = evs[0]
    e0.record(stream)
    for _ in range(a.steps):
        step_e2e()
    e1.record(stream)
    barrier_sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    peaks, peak_src = measured_peaks()
    bf16 = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    roof = None
    if kernel_ms:
        if kind == "binary" and nq <= 8:
            byts = n_local * dim / 8.0
            ach = byts / (kernel_ms * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": ach / peaks["hbm_gbs"], "traffic": None, "kernel": "k_hamming_scan",
                    "kernel_ms": kernel_ms, "bytes_per_launch": byts,
                    "peak_source": f"{peak_src} HBM copy bandwidth"}
        else:
            ops = 2.0 * nq * n_local * dim
            if kind == "float":
                peak, lab, unit = bf16, f"{peak_src} bf16 sustained", "TFLOP/s"
                prec_used = auto_precision(k, c["rerank"], c["rows"] == "f32")
                if prec_used == "tf32":
                    peak, lab = bf16 / 2.0, f"{peak_src} bf16 sustained / 2 for tf32"
            else:
                prec_used = "int8"
                peak, lab, unit = 2.0 * bf16, f"2 x {peak_src} bf16 sustained (dense int8 rate = 2 x bf16)", "TOP/s"
            ach = ops / (kernel_ms * 1e-3) / 1e12
            roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": unit, "frac": ach / peak,
                    "traffic": None, "kernel": "k_tc_filter", "kernel_ms": kernel_ms, "ops_per_launch": ops,
                    "filter_precision": prec_used, "peak_source": lab}
    in_bytes = hq.numel() * hq.element_size()
    line = {
        "metric": f"queries/sec, {a.config}: {c['desc']}", "value": nq / (ms * 1e-3), "unit": "queries/s",
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": {"float": "bf16/tf32 filter + f64 exact rerank", "int8": "s8 codes, s32 accumulate + f64 rerank",
                  "binary": "u1 codes (popcount / s8 0-1 tensor-core contraction)"}[kind],
        "data": "synthetic: TestRNG restatement on the device", "config": {
            "workload": c["desc"], "config": a.config, "N": n_total, "d": dim, "Q": nq, "k": k,
            "parallelism": f"row-shard x{world}, NCCL allgather + device merge",
            "l2_policy": "inputs larger than L2, no flush"},
        "latency_ms": {"p50": p50, "p99": p99},
        "e2e": {"value": nq / (e2e_ms * 1e-3), "unit": "queries/s", "h2d_bytes_per_step": world * in_bytes,
                "d2h_bytes_per_step": world * nq * k * 8},
        "roofline": roof, "clocks": clk,
    }
    if note:
        line["note"] = note
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ivf(a):
    """IVF search (not a BASELINE configuration): k-means lists over a mixture on one GPU, then
    K timed searches of the same query batch, device-resident (`value`) and through the host-buffer
    entry (`e2e`); recall@k against the exact flat search. Further ranks exit (replicas only)."""
    import torch

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi

    rank, world, local = env_rank()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx = va.GPUContext(va.Metal4Configuration(device=local, stream=stream.cuda_stream))
    n, dim, nq, k, nlist, nprobe = a.n, a.dim, a.nq, a.k, a.nlist, a.nprobe
    x = torch.empty((n, dim), dtype=torch.float32, device="cuda")
    q = torch.empty((nq, dim), dtype=torch.float32, device="cuda")
    _ffi.call("va_gen_mixture", ctx.handle, x.data_ptr(), n, dim, 7, 0, 256, ctypes.c_float(0.5), 0)
    _ffi.call("va_gen_mixture", ctx.handle, q.data_ptr(), nq, dim, 7, QUERY_ROW0, 256, ctypes.c_float(0.5), 0)
    cent = torch.empty((nlist, dim), dtype=torch.float32, device="cuda")
    iters = ctypes.c_int(0)
    t0 = time.perf_counter()
    _ffi.call("va_ivf_train", ctx.handle, x.data_ptr(), n, dim, nlist, a.kmeans_iters, ctypes.c_float(a.kmeans_tol),
              42, _ffi.IVF_INIT_KMEANSPP, cent.data_ptr(), ctypes.byref(iters))
    ctx.synchronize()
    t_train = time.perf_counter() - t0
    h = ctypes.c_void_p()
    _ffi.call("va_ivf_create", ctx.handle, x.data_ptr(), n, dim, cent.data_ptr(), nlist, 0, ctypes.byref(h))
    ctx.synchronize()
    ov = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    hq = q.cpu().pin_memory()
    hv = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    hi = torch.empty((nq, k), dtype=torch.int32).pin_memory()

    def step():
        _ffi.call("va_ivf_search", ctx.handle, h.value, q.data_ptr(), nq, k, nprobe, ov.data_ptr(), oi.data_ptr())

    for _ in range(a.warmup):
        step()
    ctx.synchronize()
    clocks = ClockSampler(str(local), enabled=not a.no_clocks)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(a.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / a.steps
    t0 = time.perf_counter()
    for _ in range(a.steps):
        _ffi.call("va_ivf_search_host", ctx.handle, h.value, hq.data_ptr(), nq, k, nprobe, hv.data_ptr(),
                  hi.data_ptr())
    e2e_ms = (time.perf_counter() - t0) * 1e3 / a.steps
    sizes = np.zeros(nlist, np.int64)
    _ffi.call("va_ivf_list_sizes", h.value, sizes.ctypes.data_as(ctypes.c_void_p))
    # recall@k against the exact flat search of the same rows
    db = va.Database(ctx, None, device_ptr=x.data_ptr(), n=n, dim=dim)
    ev_, ei_ = torch.empty_like(ov), torch.empty_like(oi)
    _ffi.call("va_knn_search", ctx.handle, db.handle, q.data_ptr(), nq, k, _ffi.METRIC_L2SQ, _ffi.PREC_AUTO, 0,
              ev_.data_ptr(), ei_.data_ptr())
    ctx.synchronize()
    got, ref = oi.cpu().numpy(), ei_.cpu().numpy()
    recall = float(np.mean([len(set(got[i]) & set(ref[i])) / k for i in range(nq)]))
    db.close()
    _ffi.call("va_ivf_destroy", h.value)
    line = {
        "metric": f"queries/sec, IVF search (nlist {nlist}, nprobe {nprobe}); not a BASELINE configuration",
        "value": nq / (ms * 1e-3), "unit": "queries/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None,
        "dtype": "bf16 list scan + f64 exact rerank (fp32 coarse quantizer)",
        "data": "synthetic: mixture of 256 centroids sigma 0.5 (TestRNG restatement on the device)",
        "config": {"workload": f"IVF k-NN: N={n:,} x d={dim} fp32, k-means++ then Lloyd, {nlist} lists ({iters.value} iterations, "
                               f"{t_train:.2f} s), Q={nq:,}, k={k}, nprobe={nprobe}",
                   "config": "ivf", "N": n, "d": dim, "Q": nq, "k": k, "nlist": nlist, "nprobe": nprobe,
                   f"recall@{k}_vs_exact": recall,
                   "list_rows_min_mean_max": [int(sizes.min()), float(sizes.mean()), int(sizes.max())],
                   "l2_policy": "rows (512 MB) larger than L2, no flush"},
        "e2e": {"value": nq / (e2e_ms * 1e-3), "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                "d2h_bytes_per_step": nq * k * 8},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def main():
    a = parse_args()
    if a.impl == "reference" and a.config == "ivf":
        print(json.dumps({"impl": "reference", "unavailable": "no reference arm for the ivf configuration "
                          "(not a BASELINE configuration)"}), flush=True)
    elif a.impl == "reference":
        run_reference(a)
    elif a.config == "ivf":
        run_ivf(a)
    elif a.config != "headline":
        run_config(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
