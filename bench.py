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
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "queries/sec at N=10M d=768 k=10 (1/2/4/8 B200); % tensor-pipe / HBM roofline"
QUERY_ROW0 = 1 << 31
PARITY_QUERIES = 100


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
    p.add_argument("--filter-precision", choices=["auto", "bf16", "tf32"], default="auto",
                   help="float configurations other than the headline: the filter precision (auto = the "
                        "library's PREC_AUTO choice)")
    p.add_argument("--pool-factor", type=int, default=None,
                   help="float configurations other than the headline: candidate pool = factor x k "
                        "(default: the configuration's own rerank factor)")
    p.add_argument("--rerank", type=int, default=0, help="headline: candidate-pool factor (0 = automatic)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the oracle parity check of sampled queries")
    p.add_argument("--parity-queries", type=int, default=PARITY_QUERIES)
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


# ------------------------------------------------------------------------------------------ oracle parity
# The checker leg (after timing): the search's results for a seeded sample of queries against the
# CPU oracle's exact answer over the WHOLE database. Rows are streamed from the device in chunks
# (the inputs the GPU searched); every rank checks its own shard and rank 0 merges.
PARITY_CHUNK_BYTES = 2 << 30


def parity_sample(nq: int, count: int = PARITY_QUERIES) -> np.ndarray:
    rng = np.random.default_rng(20260)
    return np.sort(rng.choice(nq, size=min(count, nq), replace=False))


def download_rows(ctx, dev_ptr: int, r0: int, r1: int, row_elems: int, dtype) -> np.ndarray:
    from vectoraccelerate_b200 import _ffi
    out = np.empty((r1 - r0, row_elems), dtype)
    isz = np.dtype(dtype).itemsize
    _ffi.call("va_buffer_download", ctx.handle, out.ctypes.data_as(ctypes.c_void_p),
              ctypes.c_void_p(dev_ptr + r0 * row_elems * isz), ctypes.c_size_t(out.nbytes))
    ctx.synchronize()
    return out


def merge_best(vals_a, ids_a, vals_b, ids_b, k: int, larger: bool):
    """Per row, the k best of two candidate lists by (value, id) (value descending when larger)."""
    v = np.concatenate([vals_a, vals_b], axis=1)
    i = np.concatenate([ids_a, ids_b], axis=1).astype(np.uint32)
    invalid = i == 0xFFFFFFFF
    key = np.where(invalid, np.inf, -v.astype(np.float64) if larger else v.astype(np.float64))
    order = np.lexsort((i.astype(np.int64), key), axis=1)[:, :k]
    return np.take_along_axis(v, order, 1), np.take_along_axis(i, order, 1)


def shard_truth(kind, ctx, db, q, k, metric, row0, n_local, dim, threads, gpu_ids, candidates=0, sq=None):
    """Oracle truth over this rank's rows [row0, row0 + n_local) (global ids), and the oracle's exact
    value of every GPU id that falls in the shard (NaN elsewhere)."""
    from oracle import oracle
    P = q.shape[0]
    larger = metric == 2 and kind == "float"
    pad = -np.inf if larger else np.inf
    tv = np.full((P, k), pad, np.float32)
    ti = np.full((P, k), 0xFFFFFFFF, np.uint32)
    gtrue = np.full(gpu_ids.shape, np.nan, np.float32)
    ptr = db.rows_ptr()
    if kind == "binary":
        row_elems, dt = dim // 32, np.uint32
    elif kind == "float" and db.dtype == 1:
        row_elems, dt = dim, np.uint16
    else:
        row_elems, dt = dim, np.float32
    chunk = max(1, PARITY_CHUNK_BYTES // (row_elems * np.dtype(dt).itemsize))
    cand_v = cand_i = None
    for r0 in range(0, n_local, chunk):
        r1 = min(n_local, r0 + chunk)
        x = download_rows(ctx, ptr, r0, r1, row_elems, dt)
        g0 = row0 + r0
        if kind == "float":
            ids, vals = oracle.knn(q, x, k, metric=metric, threads=threads, db_bf16=dt == np.uint16)
        elif kind == "binary":
            ids, d = oracle.hamming_knn(q, x, k, threads=threads)
            vals = d.astype(np.float32)
        else:
            qc = oracle.sq_perdim_quantize(q, *sq)
            xc = oracle.sq_perdim_quantize(x, *sq)
            _, _, cids, cd = oracle.int8_knn(qc, q, xc, x, candidates, 1, threads=threads)
            cvals = np.where(cd < 0, np.inf, cd).astype(np.float32)
            cids = np.where(cids == 0xFFFFFFFF, cids, cids + np.uint32(g0))
            cand_v, cand_i = (cvals, cids) if cand_v is None else merge_best(cand_v, cand_i, cvals, cids,
                                                                            candidates, False)
            ids, vals = None, None
        if ids is not None:
            ids = np.where(ids == 0xFFFFFFFF, ids, ids + np.uint32(g0))
            tv, ti = merge_best(tv, ti, vals, ids, k, larger)
        # exact values of the GPU's ids in this chunk
        inside = (gpu_ids >= g0) & (gpu_ids < row0 + r1) & (gpu_ids != 0xFFFFFFFF)
        if inside.any():
            local = np.where(inside, gpu_ids - np.uint32(g0), 0xFFFFFFFF).astype(np.uint32)
            if kind == "binary":
                for p, j in zip(*np.nonzero(inside)):
                    gtrue[p, j] = float(oracle.hamming_matrix(q[p:p + 1], x[local[p, j]:local[p, j] + 1])[0, 0])
            else:
                m = 2 if larger else (metric if kind == "float" else 0)
                rids, rvals = oracle.rerank(q, x, local, local.shape[1], metric=m, threads=threads,
                                            db_bf16=dt == np.uint16)
                for p in range(P):
                    pos = {int(a): v for a, v in zip(rids[p], rvals[p]) if int(a) != 0xFFFFFFFF}
                    for j in range(local.shape[1]):
                        if inside[p, j]:
                            gtrue[p, j] = pos[int(local[p, j])]
    if kind == "int8":
        # the int8 truth of this shard is its candidate list; reranked after the global merge
        return cand_v, cand_i, gtrue
    return tv, ti, gtrue


def int8_rerank_global(ctx, db, q, k, row0, n_local, dim, threads, cand_i):
    """Exact fp32-row rerank values of the global candidates that live in this shard (NaN elsewhere)."""
    from oracle import oracle
    vals = np.full(cand_i.shape, np.nan, np.float32)
    chunk = max(1, PARITY_CHUNK_BYTES // (dim * 4))
    ptr = db.rows_ptr()
    for r0 in range(0, n_local, chunk):
        r1 = min(n_local, r0 + chunk)
        g0 = row0 + r0
        inside = (cand_i >= g0) & (cand_i < row0 + r1) & (cand_i != 0xFFFFFFFF)
        if not inside.any():
            continue
        x = download_rows(ctx, ptr, r0, r1, dim, np.float32)
        local = np.where(inside, cand_i - np.uint32(g0), 0xFFFFFFFF).astype(np.uint32)
        rids, rvals = oracle.rerank(q, x, local, local.shape[1], metric=0, threads=threads)
        for p in range(q.shape[0]):
            pos = {int(a): v for a, v in zip(rids[p], rvals[p]) if int(a) != 0xFFFFFFFF}
            for j in range(local.shape[1]):
                if inside[p, j]:
                    vals[p, j] = pos[int(local[p, j])]
    return vals


def all_gather_host(arr: np.ndarray, world: int):
    """Every rank's copy of a host array, in rank order (on every rank)."""
    if world == 1:
        return [arr]
    import torch
    import torch.distributed as dist
    t = torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8).copy()).cuda()
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.cpu().numpy().view(arr.dtype).reshape(arr.shape) for o in out]


def oracle_sq_params(ctx, db, n_local, dim, world):
    """Per-dimension int8 parameters over the WHOLE database, computed on the host from the device
    rows (min / max per shard, combined over ranks), in the oracle's float32 formula
    (va_oracle.cpp orc_sq_perdim_params: scale = max((max - min) / 255, 1e-8))."""
    mn = np.full(dim, np.inf, np.float32)
    mx = np.full(dim, -np.inf, np.float32)
    chunk = max(1, PARITY_CHUNK_BYTES // (dim * 4))
    ptr = db.rows_ptr()
    for r0 in range(0, n_local, chunk):
        x = download_rows(ctx, ptr, r0, min(n_local, r0 + chunk), dim, np.float32)
        mn = np.minimum(mn, x.min(axis=0))
        mx = np.maximum(mx, x.max(axis=0))
    mn = np.min(np.stack(all_gather_host(mn, world)), axis=0)
    mx = np.max(np.stack(all_gather_host(mx, world)), axis=0)
    return mn, np.maximum((mx - mn) / np.float32(255.0), np.float32(1e-8)).astype(np.float32)


def oracle_parity(kind, ctx, db, queries_host, sel, final_vals, final_ids, k, metric, row0, n_local, n_total, dim,
                  world, candidates=0, sq=None):
    """Parity of the sampled queries' final results against the oracle over all ranks' rows."""
    t0 = time.perf_counter()
    threads = max(1, (os.cpu_count() or 1) // world)
    q = np.ascontiguousarray(queries_host[sel])
    gv = np.ascontiguousarray(final_vals[sel])
    gi = np.ascontiguousarray(final_ids[sel]).view(np.uint32)
    larger = metric == 2 and kind == "float"
    tv, ti, gtrue = shard_truth(kind, ctx, db, q, k, metric, row0, n_local, dim, threads, gi, candidates, sq)
    tvs, tis, gts = all_gather_host(tv, world), all_gather_host(ti, world), all_gather_host(gtrue, world)
    if kind == "int8":
        # global integer candidates, then their exact rerank on every shard
        cv, ci = tvs[0], tis[0]
        for a, b in zip(tvs[1:], tis[1:]):
            cv, ci = merge_best(cv, ci, a, b, candidates, False)
        if world > 1:
            import torch
            import torch.distributed as dist
            t = torch.from_numpy(ci.view(np.int32).copy()).cuda()
            dist.broadcast(t, 0)
            ci = t.cpu().numpy().view(np.uint32)
        rv = int8_rerank_global(ctx, db, q, k, row0, n_local, dim, threads, ci)
        rvs = all_gather_host(rv, world)
        rv = np.where(np.isnan(rvs[0]), np.nan, rvs[0])
        for a in rvs[1:]:
            rv = np.where(np.isnan(rv), a, rv)
        rv = np.where(ci == 0xFFFFFFFF, np.inf, rv)
        order = np.lexsort((ci.astype(np.int64), rv.astype(np.float64)), axis=1)[:, :k]
        tv, ti = np.take_along_axis(rv, order, 1).astype(np.float32), np.take_along_axis(ci, order, 1)
    else:
        tv, ti = tvs[0], tis[0]
        for a, b in zip(tvs[1:], tis[1:]):
            tv, ti = merge_best(tv, ti, a, b, k, larger)
    g = gts[0]
    for a in gts[1:]:
        g = np.where(np.isnan(g), a, g)
    from oracle import parity
    out = parity.summary(gi, gv, ti, tv, g)
    out["ok"] = parity.ok(out)
    out["sample"] = f"{len(sel)} seeded queries (numpy default_rng(20260)) of {queries_host.shape[0]:,}, " \
                    f"full N={n_total:,}; oracle streamed over the device rows on {threads} threads per rank"
    out["seconds"] = round(time.perf_counter() - t0, 1)
    return out


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str, enabled: bool = True):
        self.proc = None
        if not enabled:
            return
        try:
            self.f = tempfile.NamedTemporaryFile("w", suffix=".csv", delete=False)
            self.path = self.f.name
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


def make_context(va, dist, rank, world, local, stream):
    """The library context of this rank: a plain one-device context at N = 1, else one rank of an
    NCCL group (va_context_create_rank; rank 0's unique id reaches the others through the process
    group's broadcast)."""
    cfg = va.Metal4Configuration(device=local, stream=stream.cuda_stream)
    if world == 1:
        return va.GPUContext(cfg)
    nid = [va.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(nid, src=0)
    return va.GPUContext.rank(world, rank, nid[0], cfg)


def launches_per_step(ctx, world: int, precision: str):
    """Kernels of this library in one step (from the last search's certificate counts): query
    operand, filter, merge + rerank; a second pass (gather, operand, filter, merge, scatter) when
    some query was not certified; pack, unpack and shard merge on N > 1 GPUs. None on the FP32 route."""
    if precision == "fp32":
        return None
    unc, _ = ctx.last_search_stats()
    return 3 + (5 if unc else 0) + (3 if world > 1 else 0)


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
    ctx = make_context(va, dist, rank, world, local, stream)
    prec = {"bf16": va.PREC_BF16, "tf32": va.PREC_TF32, "fp32": va.PREC_FP32}[a.precision]

    # ---- database shard, generated on the device, built into a resident (sharded) va_database
    row0, n_local = ctx.shard_range(a.n) if world > 1 else (0, a.n)
    gen = torch.empty((n_local, a.dim), dtype=torch.float32, device="cuda")
    _ffi.call("va_gen_gaussian", ctx.handle, gen.data_ptr(), n_local, a.dim, 0, row0)
    if world > 1:
        db = va.ShardedDatabase(ctx, device_ptr=gen.data_ptr(), n=a.n, dim=a.dim)
    else:
        db = va.Database(ctx, None, device_ptr=gen.data_ptr(), n=n_local, dim=a.dim)
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
    final = [lv, li]

    # One step = va_knn_search over the whole database: on N > 1 GPUs each rank's library call
    # searches its shard, all-gathers packed (value, id) records over NCCL and merges on the device.
    def step_device(queries_ptr):
        _ffi.call("va_knn_search", ctx.handle, db.handle, queries_ptr, a.nq, k, va.METRIC_L2SQ, prec, a.rerank,
                  lv.data_ptr(), li.data_ptr())

    def step_e2e():
        _ffi.call("va_knn_search_host", ctx.handle, db.handle, ctypes.c_void_p(hq.data_ptr()), a.nq, k,
                  va.METRIC_L2SQ, prec, a.rerank, ctypes.c_void_p(hv.data_ptr()), ctypes.c_void_p(hi.data_ptr()))

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
    # va_knn_search_host runs on the context stream and waits; bracket with wall time too
    barrier_sync()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step_e2e()
    e2e_ms = max(e2e_ms, max_over_ranks((time.perf_counter() - t0) * 1e3 / a.steps))

    # ---- certificate counts of one step's local search, and oracle parity of sampled queries
    step_device(dq.data_ptr())
    torch.cuda.synchronize()
    lps = launches_per_step(ctx, world, a.precision)
    unc, exa = ctypes.c_int64(), ctypes.c_int64()
    _ffi.call("va_last_search_stats", ctx.handle, ctypes.byref(unc), ctypes.byref(exa))
    unc_all = all_gather_host(np.array([unc.value, exa.value], np.int64), world)
    exactness = {"uncertified_first_pass": int(sum(u[0] for u in unc_all)),
                 "exact_route": int(sum(u[1] for u in unc_all)),
                 "note": "per step, summed over ranks: queries whose first bf16 pass was not certified exact "
                         "(they take a wider tensor-core pass) and queries that took the exact SIMT route"}
    if not a.no_parity:
        vals_h = final[0].cpu().numpy()
        ids_h = final[1].cpu().numpy()
        exactness["parity"] = oracle_parity("float", ctx, db, hq.numpy(), parity_sample(a.nq, a.parity_queries),
                                            vals_h, ids_h, k, 0, row0, n_local, a.n, a.dim, world)

    db.close()
    ctx.close()
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
        "config": workload(a),
        "parallelism": f"row-shard x{world}, NCCL allgather + device merge",
        "filter_precision": a.precision,
        "exactness": exactness,
        "e2e": {"value": a.nq / (e2e_ms * 1e-3), "unit": "queries/s",
                "h2d_bytes_per_step": world * a.nq * a.dim * 4, "d2h_bytes_per_step": world * a.nq * k * 8},
        "gpu_launches": (lps * a.steps) if lps else None,
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
    """One of the other BASELINE configurations; for N > 1 the database is sharded by the library
    (N/world rows per rank, global ids = shard base + row) and each search all-gathers and merges
    inside the library call, as the headline."""
    import torch
    import torch.distributed as dist

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi

    c = CONFIGS[a.config]
    kind = c["kind"]
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    ctx = make_context(va, dist, rank, world, local, stream)
    n_total = a.n
    note = None
    row0, n_local = ctx.shard_range(n_total) if world > 1 else (0, n_total)
    dim, nq, k = a.dim, a.nq, a.k
    chunk = max(1, (4 << 30) // (4 * dim))  # fp32 generation chunks of <= 4 GiB

    def gen_f32(dst_ptr, rows, seed, r0):
        if c.get("mixture"):
            nc, sigma, norm = c["mixture"]
            _ffi.call("va_gen_mixture", ctx.handle, dst_ptr, rows, dim, seed, r0, nc, sigma, int(norm))
        else:
            _ffi.call("va_gen_gaussian", ctx.handle, dst_ptr, rows, dim, seed, r0)

    db_seed, q_seed, q_row0 = (2, 3, 0) if kind == "binary" else (0, 0, QUERY_ROW0)
    # ---- database shard (N > 1: this rank's rows of a database sharded by the library)
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
        if world > 1:
            db = va.ShardedDatabase(ctx, device_ptr=rows.data_ptr(), n=n_total, dim=dim, dtype=va.DTYPE_BF16)
        else:
            db = va.Database(ctx, None, dtype=va.DTYPE_BF16, device_ptr=rows.data_ptr(), n=n_local, dim=dim)
    elif kind in ("float", "int8"):
        rows = torch.empty((n_local, dim), dtype=torch.float32, device="cuda")
        for r in range(0, n_local, chunk):
            gen_f32(rows[r:].data_ptr(), min(chunk, n_local - r), db_seed, row0 + r)
        ctx.synchronize()
        if world > 1:
            # int8: the library codes every shard with the per-dimension range of the WHOLE
            # database (min / max all-reduced over the group)
            db = va.ShardedDatabase(ctx, device_ptr=rows.data_ptr(), n=n_total, dim=dim, kind=kind)
        elif kind == "float":
            db = va.Database(ctx, None, device_ptr=rows.data_ptr(), n=n_local, dim=dim)
        else:
            db = va.Int8Database(ctx, None, device_ptr=rows.data_ptr(), n=n_local, dim=dim)
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
        if world > 1:
            db = va.ShardedDatabase(ctx, device_ptr=rows.data_ptr(), n=n_total, dim=dim, kind="binary")
        else:
            db = va.BinaryDatabase.from_device(ctx, rows.data_ptr(), n_local, dim)
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
    cprec = {"auto": va.PREC_AUTO, "bf16": va.PREC_BF16, "tf32": va.PREC_TF32}[a.filter_precision]
    crerank = c.get("rerank", 0) if a.pool_factor is None else a.pool_factor
    final = [lv, li]

    # One step = one library call over the whole database (sharded over the ranks for N > 1).
    def search(qptr, ov, oi):
        if kind == "float":
            _ffi.call("va_knn_search", ctx.handle, db.handle, qptr, nq, k, metric, cprec, crerank, ov, oi)
        elif kind == "int8":
            _ffi.call("va_int8_knn_search", ctx.handle, db.handle, qptr, nq, k, c["candidates"], ov, oi)
        else:
            # uint32 distances land in the float array as their bit patterns
            _ffi.call("va_hamming_knn_db", ctx.handle, db.handle, qptr, nq, k, ov, oi)

    def step():
        search(dq.data_ptr(), lv.data_ptr(), li.data_ptr())

    def step_e2e():
        dq.copy_(hq, non_blocking=True)
        step()
        hv.copy_(lv, non_blocking=True)
        hi.copy_(li, non_blocking=True)

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

    # ---- certificate counts (float configurations) and oracle parity of sampled queries
    step()
    torch.cuda.synchronize()
    exactness = {}
    if kind == "float":
        unc, exa = ctypes.c_int64(), ctypes.c_int64()
        _ffi.call("va_last_search_stats", ctx.handle, ctypes.byref(unc), ctypes.byref(exa))
        tot = np.sum(np.stack(all_gather_host(np.array([unc.value, exa.value], np.int64), world)), axis=0)
        exactness = {"uncertified_first_pass": int(tot[0]), "exact_route": int(tot[1])}
    if not a.no_parity:
        vals_h = final[0].cpu().numpy()
        ids_h = final[1].cpu().numpy()
        if kind == "binary":
            vals_h = vals_h.view(np.uint32).astype(np.float32)
        sq = oracle_sq_params(ctx, db, n_local, dim, world) if kind == "int8" else None
        exactness["parity"] = oracle_parity(kind, ctx, db, hq.numpy().view(np.uint32) if kind == "binary"
                                            else hq.numpy(), parity_sample(nq, a.parity_queries), vals_h, ids_h,
                                            k, metric, row0, n_local, n_total, dim, world,
                                            candidates=c.get("candidates", 0), sq=sq)
    db.close()
    ctx.close()
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
                prec_used = (auto_precision(k, crerank, c["rows"] == "f32") if a.filter_precision == "auto"
                             else a.filter_precision)
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
            "l2_policy": "inputs larger than L2, no flush"},
        "parallelism": f"row-shard x{world}, NCCL allgather + device merge",
        "exactness": exactness,
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
    unc, exa = ctx.last_search_stats()
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
        "exactness": {"uncertified": int(unc), "exact_rescan": int(exa),
                      "note": "per step: queries whose list-scan pool the certificate could not prove exact "
                              "(they take the exact fp64 rescan of their probed lists)"},
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
