"""GPU parity of the integer search paths (int8 scalar-quantized L2 with exact rerank, Hamming on
a resident binary database) against the CPU oracle on identical seeded inputs. Needs a B200."""

import numpy as np
import pytest

from conftest import assert_knn_parity

pytestmark = pytest.mark.gpu

QROW = 1 << 31  # query streams are offset from database streams


def _true_l2(q, x, ids):
    """Exact squared L2 (fp64) of each returned id at its position."""
    valid = ids != 0xFFFFFFFF
    safe = np.where(valid, ids, 0).astype(np.int64)
    d = ((q[:, None, :].astype(np.float64) - x[safe].astype(np.float64)) ** 2).sum(-1)
    return np.where(valid, d, np.inf).astype(np.float32)


@pytest.mark.parametrize("n,dim", [(5003, 768), (3000, 100), (1000, 130)])
def test_int8_params_and_codes(ctx, oracle, n, dim):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(n, dim, 4, 64, 0.3, False)
    db = va.Int8Database(ctx, x)
    try:
        mins, scales = db.parameters()
        om, osc = oracle.sq_perdim_params(x)
        assert np.array_equal(mins, om)
        assert np.array_equal(scales, osc)
        assert np.array_equal(db.codes(), oracle.sq_perdim_quantize(x, om, osc))
    finally:
        db.close()


@pytest.mark.parametrize("n,dim,nq,k,cand", [
    (20_000, 768, 300, 10, 100),
    (20_000, 768, 300, 100, 128),
    (20_000, 768, 129, 1, 32),
    (5003, 100, 257, 10, 64),
])
def test_int8_knn(ctx, oracle, n, dim, nq, k, cand):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(n, dim, 6, 128, 0.3, False)
    q = oracle.gen_mixture(nq, dim, 6, 128, 0.3, False, row0=QROW)
    mins, scales = oracle.sq_perdim_params(x)
    xc = oracle.sq_perdim_quantize(x, mins, scales)
    qc = oracle.sq_perdim_quantize(q, mins, scales)
    oids, ovals, _, _ = oracle.int8_knn(qc, q, xc, x, cand, k)
    db = va.Int8Database(ctx, x)
    try:
        vals, ids = db.search(q, k, cand)
    finally:
        db.close()
    assert_knn_parity(ids, vals, oids, ovals, _true_l2(q, x, ids))


def test_int8_knn_given_range_and_id_base(ctx, oracle):
    """Codes from a range wider than the shard's own (the global range of a sharded database);
    ids carry the shard's base."""
    import vectoraccelerate_b200 as va
    n, dim, nq, k, cand = 6000, 256, 200, 10, 64
    x = oracle.gen_mixture(n, dim, 8, 32, 0.3, False)
    q = oracle.gen_mixture(nq, dim, 8, 32, 0.3, False, row0=QROW)
    om, osc = oracle.sq_perdim_params(x)
    mn = om - 0.5
    mx = om + osc * 255.0 + 0.25
    sc = np.maximum((mx - mn) / np.float32(255.0), np.float32(1e-8)).astype(np.float32)
    xc = oracle.sq_perdim_quantize(x, mn, sc)
    qc = oracle.sq_perdim_quantize(q, mn, sc)
    oids, ovals, _, _ = oracle.int8_knn(qc, q, xc, x, cand, k)
    db = va.Int8Database(ctx, x, id_base=1000, mins=mn, maxs=mx)
    try:
        gm, gs = db.parameters()
        assert np.array_equal(gm, mn) and np.array_equal(gs, sc)
        vals, ids = db.search(q, k, cand)
    finally:
        db.close()
    ids0 = ids - np.uint32(1000)
    assert_knn_parity(ids0, vals, oids, ovals, _true_l2(q, x, ids0))


def test_int8_errors(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(1000, 64, 1)
    db = va.Int8Database(ctx, x)
    try:
        with pytest.raises(va.InvalidInput):
            db.search(x[:4], 10, 5)      # candidates < k
        with pytest.raises(va.InvalidInput):
            db.search(x[:4, :32], 10, 32)  # wrong dimension
    finally:
        db.close()


@pytest.mark.parametrize("n,bits,nq,k", [
    (20_000, 1024, 300, 100),
    (20_000, 1024, 129, 1),
    (5003, 96, 257, 10),
    (4000, 64, 64, 128),
    (3000, 1000, 100, 16),
])
def test_hamming_db_knn(ctx, oracle, n, bits, nq, k):
    import vectoraccelerate_b200 as va
    x = oracle.binary_quantize(oracle.gen_gaussian(n, bits, 2))
    q = oracle.binary_quantize(oracle.gen_gaussian(nq, bits, 2, row0=QROW))
    oi, od = oracle.hamming_knn(q, x, k)
    db = va.BinaryDatabase(ctx, x, bits)
    try:
        gd, gi = db.search(q, k)
    finally:
        db.close()
    assert np.array_equal(gd, od)
    assert np.array_equal(gi, oi)  # integer distances: the (distance, id) order is exact


def test_hamming_db_duplicates_and_base(ctx, oracle):
    """Massive ties (every code repeated 50 times): the (distance, id) order must hold across
    row splits; ids carry the base."""
    import vectoraccelerate_b200 as va
    base = oracle.binary_quantize(oracle.gen_gaussian(400, 256, 9))
    x = np.repeat(base, 50, axis=0)
    q = base[:37].copy()
    oi, od = oracle.hamming_knn(q, x, 128)
    db = va.BinaryDatabase(ctx, x, 256, id_base=7)
    try:
        gd, gi = db.search(q, 128)
    finally:
        db.close()
    assert np.array_equal(gd, od)
    assert np.array_equal(gi - np.uint32(7), oi)


@pytest.mark.parametrize("n,bits,nq,k", [
    (200_000, 1024, 1, 100),
    (200_000, 1024, 8, 100),
    (50_000, 512, 3, 128),
    (50_000, 256, 5, 1),
    (30_001, 128, 2, 64),
    (5003, 96, 1, 10),      # 3 words: no packed scan, the expanded tensor-core route
])
def test_hamming_db_small_batch(ctx, oracle, n, bits, nq, k):
    """Small batches take the HBM-bound scan over the packed codes."""
    import vectoraccelerate_b200 as va
    x = oracle.binary_quantize(oracle.gen_gaussian(n, bits, 2))
    q = oracle.binary_quantize(oracle.gen_gaussian(nq, bits, 3, row0=QROW))
    oi, od = oracle.hamming_knn(q, x, k)
    db = va.BinaryDatabase(ctx, x, bits, id_base=11)
    try:
        gd, gi = db.search(q, k)
    finally:
        db.close()
    assert np.array_equal(gd, od)
    assert np.array_equal(gi - np.uint32(11), oi)


def test_hamming_db_small_batch_ties(ctx, oracle):
    """Every code 300 times in a row: distance-0 runs force repeated buffer compactions; the
    (distance, id) order must survive them."""
    import vectoraccelerate_b200 as va
    base = oracle.binary_quantize(oracle.gen_gaussian(200, 1024, 5))
    x = np.repeat(base, 300, axis=0)
    q = base[[3, 150, 199]].copy()
    oi, od = oracle.hamming_knn(q, x, 128)
    db = va.BinaryDatabase(ctx, x, 1024)
    try:
        gd, gi = db.search(q, 128)
        gd1, gi1 = db.search(q[:1], 128)
    finally:
        db.close()
    assert np.array_equal(gd, od) and np.array_equal(gi, oi)
    assert np.array_equal(gd1, od[:1]) and np.array_equal(gi1, oi[:1])


@pytest.mark.parametrize("chunk", [5000, 256])
def test_hamming_db_chunked_expansion(ctx, oracle, chunk):
    """Batches over a database expanded chunk by chunk (the route of databases whose 0/1
    expansion does not fit): same results, ties across chunk boundaries included."""
    import vectoraccelerate_b200 as va
    base = oracle.binary_quantize(oracle.gen_gaussian(3000, 512, 12))
    x = np.concatenate([base, base[:2000]])  # duplicates in different chunks
    q = oracle.binary_quantize(oracle.gen_gaussian(150, 512, 13, row0=QROW))
    q[:5] = base[[0, 100, 1999, 2500, 2999]]
    oi, od = oracle.hamming_knn(q, x, 64)
    db = va.BinaryDatabase(ctx, x, 512, id_base=3)
    try:
        db.set_chunk_rows(chunk)
        gd, gi = db.search(q, 64)
    finally:
        db.close()
    assert np.array_equal(gd, od)
    assert np.array_equal(gi - np.uint32(3), oi)
