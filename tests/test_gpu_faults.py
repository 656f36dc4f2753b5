"""Failure paths on a B200, made without faulting the GPU.

* A bounded device wait that runs out: a test hook stops the filter's MMA issuer after a few
  tiles (VA_TC_TEST_STALL_TILES), so the epilogue's wait for the next accumulator has nothing to
  wait for and expires after a short limit (VA_TC_WAIT_LIMIT_MS). The kernel drains the copies
  and MMAs it already issued, frees its TMEM and returns; va_synchronize reports VA_ERR_TIMEOUT
  (the reference's error path: a command buffer error becomes computeFailed,
  Core/Metal4Context.swift:406-409), and the same context then searches correctly.
* Allocation failures: requests far beyond the device's memory give VA_ERR_OOM
  (VectorError.bufferAllocationFailed) and leave the free memory as it was.
"""

import os

import numpy as np
import pytest

from test_gpu_parity import _check

pytestmark = pytest.mark.gpu


def test_bounded_filter_wait_expires_and_the_context_recovers(oracle):
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(4)
    x = rng.standard_normal((40_000, 256)).astype(np.float32)
    q = rng.standard_normal((300, 256)).astype(np.float32)
    ctx = va.GPUContext()
    try:
        db = va.Database(ctx, x)
        os.environ["VA_TC_TEST_STALL_TILES"] = "3"
        os.environ["VA_TC_WAIT_LIMIT_MS"] = "50"
        try:
            with pytest.raises(va.Timeout, match="bounded device-side wait expired"):
                va.knn_search_host(ctx, db, q, 10, va.METRIC_L2SQ, va.PREC_BF16)
        finally:
            del os.environ["VA_TC_TEST_STALL_TILES"]
            del os.environ["VA_TC_WAIT_LIMIT_MS"]
        # the error word was consumed: the same context and database search correctly again
        ctx.synchronize()
        vals, ids = va.knn_search_host(ctx, db, q, 10, va.METRIC_L2SQ, va.PREC_BF16)
        _check(oracle, q, x, 10, 0, vals, ids)
        db.close()
    finally:
        ctx.close()
    # and a fresh context too
    ctx = va.GPUContext()
    try:
        db = va.Database(ctx, x)
        vals, ids = va.knn_search_host(ctx, db, q, 10)
        _check(oracle, q, x, 10, 0, vals, ids)
        db.close()
    finally:
        ctx.close()


def test_allocation_failures_report_oom_and_leak_nothing():
    import ctypes

    import torch

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi
    torch.cuda.init()
    ctx = va.GPUContext()
    rows = torch.zeros(16, dtype=torch.float32, device="cuda")

    def failing_calls():
        p = ctypes.c_void_p()
        with pytest.raises(va.BufferAllocationFailed):
            _ffi.call("va_buffer_alloc", ctx.handle, ctypes.c_size_t(1 << 50), ctypes.byref(p))
        assert p.value is None
        # a database larger than the device: its partial allocations are released
        h = ctypes.c_void_p()
        with pytest.raises(va.BufferAllocationFailed):
            _ffi.call("va_db_create", ctx.handle, rows.data_ptr(), 1, 4_000_000_000, 4096, 0, 0, ctypes.byref(h))
        assert h.value is None
        with pytest.raises(va.BufferAllocationFailed):
            _ffi.call("va_host_alloc", ctx.handle, ctypes.c_size_t(1 << 52), ctypes.byref(p))
        ctx.synchronize()
        torch.cuda.synchronize()

    try:
        failing_calls()  # first round: lazy driver and runtime initialisation may take memory
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            failing_calls()
        assert torch.cuda.mem_get_info()[0] == free0, "failed allocations changed the device's free memory"
    finally:
        ctx.close()
