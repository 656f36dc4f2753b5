"""The allocation-free search entry point (va_knn_search_noalloc).

It exists for callers that must not allocate device memory at search time: processes that give
all free device memory to their own pool when they start, callers whose device memory belongs to
another allocator, and latency-bound paths that cannot afford an allocation's implicit device
synchronisation. It uses one fixed device array for its scratch instead of cudaMalloc.

The test calls it through the C ABI twice in a row and compares each result with va_knn_search
on the same inputs (ids exactly, distances within the suite's 1e-4 relative tolerance), checks
that the calls leave the device's free memory unchanged, and that oversized batches are rejected.
This file is collected last so a failure here cannot hide the rest of the suite.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _search(ctx, db, dq, nq, k, fn, metric=0):
    import torch

    from vectoraccelerate_b200 import _ffi
    ov = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    _ffi.call(fn, ctx.handle, db.handle, dq.data_ptr(), nq, k, metric, 0, 0, ov.data_ptr(), oi.data_ptr())
    ctx.synchronize()
    return ov.cpu().numpy(), oi.cpu().numpy().view(np.uint32)


def test_noalloc_matches_search_on_two_calls():
    import torch

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi

    torch.cuda.init()
    rng = np.random.default_rng(7)
    x = rng.standard_normal((20_000, 256)).astype(np.float32)
    ctx = va.GPUContext()
    try:
        db = va.Database(ctx, x)
        for metric, nq, k in ((va.METRIC_L2SQ, 200, 10), (va.METRIC_IP, 33, 16)):
            q = torch.from_numpy(rng.standard_normal((nq, 256)).astype(np.float32)).cuda()
            ref_v, ref_i = _search(ctx, db, q, nq, k, "va_knn_search", metric)
            free = []
            for _ in range(2):
                v, i = _search(ctx, db, q, nq, k, "va_knn_search_noalloc", metric)
                free.append(torch.cuda.mem_get_info()[0])
                assert np.array_equal(i, ref_i)
                np.testing.assert_allclose(v, ref_v, rtol=1e-4, atol=1e-6)
            assert free[0] == free[1], "the allocation-free search changed the device's free memory"
        # a batch whose scratch exceeds the fixed array is refused, naming the bytes needed
        big = torch.zeros((40_000, 256), dtype=torch.float32, device="cuda")
        ov = torch.empty((40_000, 10), dtype=torch.float32, device="cuda")
        oi = torch.empty((40_000, 10), dtype=torch.int32, device="cuda")
        with pytest.raises(va.InvalidInput, match="bytes of scratch"):
            _ffi.call("va_knn_search_noalloc", ctx.handle, db.handle, big.data_ptr(), 40_000, 10, 0, 0, 0,
                      ov.data_ptr(), oi.data_ptr())
        # the exact FP32 route allocates, so it is refused here
        with pytest.raises(va.InvalidInput, match="tensor-core route only"):
            _ffi.call("va_knn_search_noalloc", ctx.handle, db.handle, big.data_ptr(), 4, 10, 0, va.PREC_FP32, 0,
                      ov.data_ptr(), oi.data_ptr())
        db.close()
    finally:
        ctx.close()


def test_noalloc_symbol_is_exported():
    from vectoraccelerate_b200 import _ffi
    assert hasattr(_ffi.load(), "va_knn_search_noalloc")
    assert isinstance(_ffi.load().va_knn_search_noalloc, ctypes._CFuncPtr)
