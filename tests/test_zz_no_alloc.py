"""The allocation-free search entry point (va_knn_search_noalloc).

It exists for callers that must not allocate device memory at search time: processes that give
all free device memory to their own pool when they start, callers whose device memory belongs to
another allocator, and latency-bound paths that cannot afford an allocation's implicit device
synchronisation. It uses one fixed device array for its scratch instead of cudaMalloc.

The test calls it through the C ABI twice in a row and compares each result with va_knn_search
on the same inputs (ids exactly, distances within the suite's 1e-4 relative tolerance) and with
the CPU oracle (the suite's parity rule), checks that the calls leave the device's free memory as
it was before the first of them, and that oversized batches and allocating routes are rejected.
This file is collected last so a failure here cannot hide the rest of the suite.
"""

import ctypes

import numpy as np
import pytest

from conftest import assert_knn_parity

pytestmark = pytest.mark.gpu


def _search(ctx, db, dq, nq, k, fn, metric=0, precision=0):
    import torch

    from vectoraccelerate_b200 import _ffi
    ov = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    oi = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    _ffi.call(fn, ctx.handle, db.handle, dq.data_ptr(), nq, k, metric, precision, 0, ov.data_ptr(), oi.data_ptr())
    ctx.synchronize()
    return ov.cpu().numpy(), oi.cpu().numpy().view(np.uint32)


def _oracle_parity(oracle, q, x, k, metric, vals, ids):
    tids, tvals = oracle.knn(q, x, k, metric=metric)
    rids, rvals = oracle.rerank(q, x, ids, k, metric=metric)
    gt = np.empty_like(vals)
    for r in range(ids.shape[0]):
        pos = {int(i): v for i, v in zip(rids[r], rvals[r])}
        gt[r] = [pos[int(i)] for i in ids[r]]
    assert_knn_parity(ids, vals, tids, tvals, gt)


# (metric, queries, k, dimension, precision): the default pool; a 3k pool whose 128-entry lists do
# not fit the fixed array (the lists shrink to 64 entries); k = 50 with 256 queries; d = 8 with an
# explicit bf16 pass (the certificate sends what bf16 keys cannot separate to the exact route).
CASES = [(0, 200, 10, 256, 0), (2, 33, 16, 256, 0), (0, 64, 30, 256, 0), (0, 256, 50, 256, 0), (0, 40, 10, 8, 3)]


def test_noalloc_matches_search_and_oracle_on_two_calls(oracle):
    import torch

    import vectoraccelerate_b200 as va

    torch.cuda.init()
    rng = np.random.default_rng(7)
    ctx = va.GPUContext()
    try:
        dbs = {}
        for d in sorted({c[3] for c in CASES}):
            x = rng.standard_normal((20_000, d)).astype(np.float32)
            dbs[d] = (x, va.Database(ctx, x))
        for metric, nq, k, d, prec in CASES:
            x, db = dbs[d]
            qh = rng.standard_normal((nq, d)).astype(np.float32)
            q = torch.from_numpy(qh).cuda()
            ref_v, ref_i = _search(ctx, db, q, nq, k, "va_knn_search", metric, prec)
            torch.cuda.synchronize()
            free = [torch.cuda.mem_get_info()[0]]
            for _ in range(2):
                v, i = _search(ctx, db, q, nq, k, "va_knn_search_noalloc", metric, prec)
                free.append(torch.cuda.mem_get_info()[0])
                assert np.array_equal(i, ref_i), (metric, nq, k, d)
                np.testing.assert_allclose(v, ref_v, rtol=1e-4, atol=1e-6)
                _oracle_parity(oracle, qh, x, k, metric, v, i)
            assert free[0] == free[1] == free[2], f"the allocation-free search changed the free memory: {free}"
        _, db = dbs[256]
        # a batch whose scratch exceeds the fixed array at every list size is refused, naming the bytes
        big = torch.zeros((40_000, 256), dtype=torch.float32, device="cuda")
        ov = torch.empty((40_000, 10), dtype=torch.float32, device="cuda")
        oi = torch.empty((40_000, 10), dtype=torch.int32, device="cuda")
        with pytest.raises(va.InvalidInput, match="bytes of scratch"):
            _ffi_call("va_knn_search_noalloc", ctx.handle, db.handle, big.data_ptr(), 40_000, 10, 0, 0, 0,
                      ov.data_ptr(), oi.data_ptr())
        # the exact FP32 route allocates, so it is refused here, explicitly or under AUTO (d <= 16)
        with pytest.raises(va.InvalidInput, match="tensor-core route only"):
            _ffi_call("va_knn_search_noalloc", ctx.handle, db.handle, big.data_ptr(), 4, 10, 0, va.PREC_FP32, 0,
                      ov.data_ptr(), oi.data_ptr())
        with pytest.raises(va.Unsupported, match="exact FP32 route"):
            _ffi_call("va_knn_search_noalloc", ctx.handle, dbs[8][1].handle, big.data_ptr(), 4, 10, 0, 0, 0,
                      ov.data_ptr(), oi.data_ptr())
        for _, db in dbs.values():
            db.close()
    finally:
        ctx.close()


def _ffi_call(*args):
    from vectoraccelerate_b200 import _ffi
    _ffi.call(*args)


def test_noalloc_symbol_is_exported():
    from vectoraccelerate_b200 import _ffi
    assert hasattr(_ffi.load(), "va_knn_search_noalloc")
    assert isinstance(_ffi.load().va_knn_search_noalloc, ctypes._CFuncPtr)
