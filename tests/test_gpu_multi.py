"""The sharded search through the C ABI on two or more B200s (skipped on one GPU).

A multi-device context (one process, every device) and rank contexts (one process per GPU, an
NCCL unique id shared out of band) shard the database by rows; every device searches its shard,
one all-gather of packed (value, id) records and a device merge give the global top k, which
must equal the oracle's exact answer over the WHOLE database (the single-GPU search's contract,
CPUTopK.swift:62-79). Failure paths: a rank that never joins, and a rank that leaves between
two searches, end the others' waits with a bounded error (NVLS off in those children)."""

import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from test_gpu_parity import _check

pytestmark = pytest.mark.gpu


def _ndev():
    import torch
    return torch.cuda.device_count()


needs2 = pytest.mark.skipif("_ndev() < 2", reason="needs two GPUs")


@needs2
@pytest.mark.parametrize("metric", [0, 1, 2])
def test_multi_device_context_float(oracle, metric):
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(30 + metric)
    x = rng.standard_normal((30_001, 128)).astype(np.float32)
    q = rng.standard_normal((300, 128)).astype(np.float32)
    ctx = va.GPUContext.multi([0, 1])
    try:
        assert ctx.group() == (2, 0, 2)
        assert ctx.shard_range(30_001, 1) == (15_000, 15_001)
        db = va.ShardedDatabase(ctx, x)
        vals, ids = va.knn_search_host(ctx, db, q, 10, metric)
        _check(oracle, q, x, 10, metric, vals, ids)
        db.close()
    finally:
        ctx.close()


@needs2
def test_multi_device_context_int8_and_binary(oracle):
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(8)
    x = rng.standard_normal((20_000, 96)).astype(np.float32)
    q = rng.standard_normal((64, 96)).astype(np.float32)
    ctx = va.GPUContext.multi([0, 1])
    try:
        db = va.ShardedDatabase(ctx, x, kind="int8")
        mins, scales = oracle.sq_perdim_params(x)  # the range of the WHOLE database
        qc, xc = oracle.sq_perdim_quantize(q, mins, scales), oracle.sq_perdim_quantize(x, mins, scales)
        tids, tvals, _, _ = oracle.int8_knn(qc, q, xc, x, 200, 20)
        dq = ctx.get_buffer_for(q)
        ov = ctx.get_buffer(64 * 20 * 4, np.float32, (64, 20))
        oi = ctx.get_buffer(64 * 20 * 4, np.uint32, (64, 20))
        va._ffi.call("va_int8_knn_search", ctx.handle, db.handle, dq.ptr, 64, 20, 200, ov.ptr, oi.ptr)
        np.testing.assert_array_equal(oi.download(), tids)
        np.testing.assert_allclose(ov.download(), tvals, rtol=1e-6)
        db.close()
        codes = oracle.binary_quantize(rng.standard_normal((40_000, 256)).astype(np.float32))
        qcodes = oracle.binary_quantize(rng.standard_normal((32, 256)).astype(np.float32))
        bdb = va.ShardedDatabase(ctx, codes, kind="binary")
        tids, tds = oracle.hamming_knn(qcodes, codes, 16)
        dq = ctx.get_buffer_for(qcodes)
        od = ctx.get_buffer(32 * 16 * 4, np.uint32, (32, 16))
        oi = ctx.get_buffer(32 * 16 * 4, np.uint32, (32, 16))
        va._ffi.call("va_hamming_knn_db", ctx.handle, bdb.handle, dq.ptr, 32, 16, od.ptr, oi.ptr)
        np.testing.assert_array_equal(oi.download(), tids)
        np.testing.assert_array_equal(od.download(), tds)
        bdb.close()
    finally:
        ctx.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank, world, nid, mode, out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch  # noqa: F401  (loads the same libnccl.so.2 as the process that made the id)

    import vectoraccelerate_b200 as va
    t0 = time.time()
    try:
        if mode == "never_joins" and rank == 1:
            out.put((rank, "absent", 0.0))
            return
        ctx = va.GPUContext.rank(world, rank, nid, va.Metal4Configuration(device=rank, timeout_ms=8000))
        rng = np.random.default_rng(77)
        x = rng.standard_normal((50_001, 64)).astype(np.float32)
        q = rng.standard_normal((100, 64)).astype(np.float32)
        r0, cnt = ctx.shard_range(len(x))
        if mode == "int8":
            # each rank's rows on its own device; the library all-reduces the coding range
            import torch
            rows = torch.from_numpy(x[r0:r0 + cnt]).to(f"cuda:{rank}")
            db = va.ShardedDatabase(ctx, device_ptr=rows.data_ptr(), n=len(x), dim=64, kind="int8")
            dq = ctx.get_buffer_for(q)
            ov = ctx.get_buffer(100 * 10 * 4, np.float32, (100, 10))
            oi = ctx.get_buffer(100 * 10 * 4, np.uint32, (100, 10))
            va._ffi.call("va_int8_knn_search", ctx.handle, db.handle, dq.ptr, 100, 10, 100, ov.ptr, oi.ptr)
            out.put((rank, (ov.download(), oi.download()), 0.0))
            db.close()
            ctx.close()
            return
        db = va.ShardedDatabase(ctx, x[r0:r0 + cnt], n=len(x), dim=64)
        vals, ids = va.knn_search_host(ctx, db, q, 10)
        if mode == "leaves" and rank == 1:
            # between two searches: nothing of this rank is in flight; it releases its
            # communicator and exits without joining the next collective
            db.close()
            ctx.close()
            out.put((rank, "left", 0.0))
            return
        if mode == "leaves":
            t0 = time.time()
            try:
                va.knn_search_host(ctx, db, q, 10)
                out.put((rank, "completed", time.time() - t0))
            except va.VectorError as e:
                out.put((rank, type(e).__name__, time.time() - t0))
            return
        out.put((rank, (vals, ids), 0.0))
        db.close()
        ctx.close()
    except va.VectorError as e:
        out.put((rank, type(e).__name__, time.time() - t0))


def _run_ranks(mode, world=2):
    import vectoraccelerate_b200 as va
    nid = va.nccl_unique_id()
    c = mp.get_context("spawn")
    out = c.Queue()
    procs = [c.Process(target=_rank_worker, args=(r, world, nid, mode, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, what, secs = out.get(timeout=180)
            res[r] = (what, secs)
    finally:
        # a rank that never reports must not keep the test process (and its exit) waiting
        for p in procs:
            p.join(timeout=60 if len(res) == world else 1)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    return res


@needs2
def test_rank_contexts_match_the_oracle(oracle):
    res = _run_ranks("ok")
    rng = np.random.default_rng(77)
    x = rng.standard_normal((50_001, 64)).astype(np.float32)
    q = rng.standard_normal((100, 64)).astype(np.float32)
    for r in (0, 1):
        vals, ids = res[r][0]
        _check(oracle, q, x, 10, 0, vals, ids)


@needs2
def test_rank_contexts_int8_match_the_oracle(oracle):
    # int8 database sharded over rank contexts from device rows: both range reductions in one
    # NCCL group (a non-blocking communicator takes one call at a time)
    res = _run_ranks("int8")
    rng = np.random.default_rng(77)
    x = rng.standard_normal((50_001, 64)).astype(np.float32)
    q = rng.standard_normal((100, 64)).astype(np.float32)
    mins, scales = oracle.sq_perdim_params(x)
    qc, xc = oracle.sq_perdim_quantize(q, mins, scales), oracle.sq_perdim_quantize(x, mins, scales)
    tids, tvals, _, _ = oracle.int8_knn(qc, q, xc, x, 100, 10)
    for r in (0, 1):
        vals, ids = res[r][0]
        np.testing.assert_array_equal(ids, tids)
        np.testing.assert_allclose(vals, tvals, rtol=1e-6)


@needs2
def test_rank_that_never_joins_gives_a_bounded_timeout():
    res = _run_ranks("never_joins")
    what, secs = res[0]
    assert what in ("Timeout", "CollectiveFailed"), what
    assert secs < 60


@needs2
def test_rank_that_leaves_between_searches_gives_a_bounded_error():
    res = _run_ranks("leaves")
    what, secs = res[0]
    assert what in ("Timeout", "CollectiveFailed"), what
    assert secs < 60
