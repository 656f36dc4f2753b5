"""Ingestion on the device (append with geometric growth, update, compaction) against databases
built in one piece and the oracle. Needs a B200."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

QROW = 1 << 31


def _search(ctx, db, q, k, metric=0, precision=0):
    import vectoraccelerate_b200 as va
    return va.knn_search_host(ctx, db, q, k, metric, precision)


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_append_in_pieces_equals_one_piece(ctx, oracle, metric):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(5000, 100, 81, 16, 0.3, metric == 1)
    q = oracle.gen_mixture(33, 100, 81, 16, 0.3, metric == 1, row0=QROW)
    db = va.Database(ctx, x[:700])
    try:
        for a, b in [(700, 701), (701, 2000), (2000, 2255), (2255, 5000)]:
            db.append(x[a:b])
        assert db.n == 5000
        for precision in (1, 2, 3):
            vals, ids = _search(ctx, db, q, 10, metric, precision)
            tids, tvals = oracle.knn(q, x, 10, metric=metric)
            assert np.array_equal(ids, tids)
            np.testing.assert_allclose(vals, tvals, rtol=1e-4, atol=1e-6)
    finally:
        db.close()


def test_update_and_compact(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(3000, 64, 83)
    q = oracle.gen_gaussian(20, 64, 84, row0=QROW)
    db = va.Database(ctx, x)
    try:
        x2 = x.copy()
        x2[1000:1010] = oracle.gen_gaussian(10, 64, 85)
        db.update(1000, x2[1000:1010])
        vals, ids = _search(ctx, db, q, 10, precision=3)
        tids, _ = oracle.knn(q, x2, 10)
        assert np.array_equal(ids, tids)
        keep = np.ones(3000, bool)
        keep[::3] = False
        new_slot = db.compact(keep)
        assert db.n == 2000 and new_slot[0] == -1 and new_slot[1] == 0 and new_slot[2999] == 1999
        for precision in (1, 3):
            vals, ids = _search(ctx, db, q, 10, precision=precision)
            tids, tvals = oracle.knn(q, x2[keep], 10)
            assert np.array_equal(ids, tids)
        db.append(x[:5])  # growth after a compaction
        vals, ids = _search(ctx, db, q, 10, precision=3)
        tids, _ = oracle.knn(q, np.concatenate([x2[keep], x[:5]]), 10)
        assert np.array_equal(ids, tids)
    finally:
        db.close()


def test_int8_and_binary_append(ctx, oracle):
    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi
    x = oracle.gen_mixture(6000, 128, 86, 32, 0.3, False)
    q = oracle.gen_mixture(40, 128, 86, 32, 0.3, False, row0=QROW)
    mins, scales = oracle.sq_perdim_params(x)
    maxs = (mins + scales * np.float32(255.0)).astype(np.float32)
    idb = va.Int8Database(ctx, x[:1000], mins=mins, maxs=maxs)
    try:
        _ffi.call("va_db_append", ctx.handle, idb.handle, x[1000:].ctypes.data_as(_ffi.ctypes.c_void_p), 0, 5000)
        ctx.synchronize()
        idb.n = 6000
        gm, gs = idb.parameters()
        xc = oracle.sq_perdim_quantize(x, gm, gs)
        qc = oracle.sq_perdim_quantize(q, gm, gs)
        oids, ovals, _, _ = oracle.int8_knn(qc, q, xc, x, 64, 10)
        vals, ids = idb.search(q, 10, 64)
        assert np.array_equal(ids, oids)
    finally:
        idb.close()
    codes = oracle.binary_quantize(oracle.gen_gaussian(4000, 256, 87))
    qb = oracle.binary_quantize(oracle.gen_gaussian(20, 256, 88, row0=QROW))
    bdb = va.BinaryDatabase(ctx, codes[:100], 256)
    try:
        bdb.search(qb, 16)  # builds the resident expansion before the append
        _ffi.call("va_db_append", ctx.handle, bdb.handle, codes[100:].ctypes.data_as(_ffi.ctypes.c_void_p), 0, 3900)
        ctx.synchronize()
        gd, gi = bdb.search(qb, 16)
        oi, od = oracle.hamming_knn(qb, codes, 16)
        assert np.array_equal(gi, oi) and np.array_equal(gd, od)
        gd1, gi1 = bdb.search(qb[:1], 16)  # packed-code scan sees the appended rows too
        assert np.array_equal(gi1, oi[:1])
    finally:
        bdb.close()
