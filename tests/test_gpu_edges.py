"""GPU parity at the edges of the fused search: zero vectors under cosine, the largest supported
dimension, one-dimensional rows, a database of one repeated row (every distance ties), queries
equal to database rows, large magnitudes, and k equal to the database size. Needs a B200."""

import numpy as np
import pytest

from conftest import assert_knn_parity

pytestmark = pytest.mark.gpu

QROW = 1 << 31


def _search(ctx, x, q, k, metric=0, precision=0, rerank=0):
    import vectoraccelerate_b200 as va
    db = va.Database(ctx, x)
    try:
        return va.knn_search_host(ctx, db, q, k, metric, precision, rerank)
    finally:
        db.close()


def _true_vals(oracle, q, x, ids, metric):
    """Oracle truth values of the returned ids at their positions (fp64, one rounding)."""
    out = np.empty(ids.shape, np.float32)
    for r in range(ids.shape[0]):
        valid = ids[r] != 0xFFFFFFFF
        m = (oracle.matrix(q[r:r + 1], x[ids[r][valid].astype(np.int64)], metric, flag=metric == 1)
             if valid.any() else None)
        out[r] = np.inf if metric != 2 else -np.inf
        if m is not None:
            out[r][valid] = m[0]
    return out


@pytest.mark.parametrize("precision", [1, 2, 3], ids=["fp32", "tf32", "bf16"])
def test_cosine_zero_vectors(ctx, oracle, precision):
    """A zero row or query has similarity 0 with everything (distance 1), as the reference's
    AccelerateFallback defines it."""
    x = oracle.gen_gaussian(500, 64, 41)
    x[[3, 77, 499]] = 0.0
    q = oracle.gen_gaussian(9, 64, 42, row0=QROW)
    q[4] = 0.0
    vals, ids = _search(ctx, x, q, 20, metric=1, precision=precision)
    tids, tvals = oracle.knn(q, x, 20, metric=1)
    assert_knn_parity(ids, vals, tids, tvals, _true_vals(oracle, q, x, ids, 1))
    assert np.allclose(vals[4], 1.0)  # the zero query: every distance is 1, ids 0..19 by the tie rule
    assert np.array_equal(ids[4], np.arange(20, dtype=np.uint32))


@pytest.mark.parametrize("metric", [0, 2])
def test_max_dimension(ctx, oracle, metric):
    x = oracle.gen_gaussian(3000, 4096, 43)
    q = oracle.gen_gaussian(40, 4096, 44, row0=QROW)
    for precision in (1, 3):
        vals, ids = _search(ctx, x, q, 10, metric=metric, precision=precision)
        tids, tvals = oracle.knn(q, x, 10, metric=metric)
        assert_knn_parity(ids, vals, tids, tvals, _true_vals(oracle, q, x, ids, metric))


def test_one_dimensional_rows(ctx, oracle):
    """Automatic precision takes the exact FP32 route at d <= 16: reduced-precision keys cannot
    separate neighbours 1/N apart on a line (an explicit BF16/TF32 request is exact only when the
    true top k fall inside its candidate pool, which they do not here)."""
    x = oracle.gen_gaussian(2000, 1, 45)
    q = oracle.gen_gaussian(33, 1, 46, row0=QROW)
    for precision in (0, 1):
        vals, ids = _search(ctx, x, q, 7, precision=precision)
        tids, tvals = oracle.knn(q, x, 7)
        assert_knn_parity(ids, vals, tids, tvals, _true_vals(oracle, q, x, ids, 0))


@pytest.mark.parametrize("precision", [1, 2, 3], ids=["fp32", "tf32", "bf16"])
def test_all_rows_identical(ctx, oracle, precision):
    """Every distance ties: the result is ids 0..k-1 in order."""
    x = np.repeat(oracle.gen_gaussian(1, 48, 47), 3000, axis=0)
    q = oracle.gen_gaussian(5, 48, 48, row0=QROW)
    vals, ids = _search(ctx, x, q, 25, precision=precision)
    assert np.array_equal(ids, np.tile(np.arange(25, dtype=np.uint32), (5, 1)))
    tids, tvals = oracle.knn(q, x, 25)
    assert np.allclose(vals, tvals, rtol=1e-5)


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_queries_equal_rows(ctx, oracle, metric):
    x = oracle.gen_mixture(4000, 96, 49, 16, 0.3, metric == 1)
    q = x[[0, 17, 1999, 3999]].copy()
    vals, ids = _search(ctx, x, q, 5, metric=metric, precision=3)
    tids, tvals = oracle.knn(q, x, 5, metric=metric)
    assert_knn_parity(ids, vals, tids, tvals, _true_vals(oracle, q, x, ids, metric))
    if metric == 0:
        assert np.array_equal(ids[:, 0], np.array([0, 17, 1999, 3999], np.uint32))
        assert np.all(vals[:, 0] == 0.0)


def test_large_magnitudes(ctx, oracle):
    """Rows scaled by 1e3: the bf16 filter keys stay finite and the exact rerank restores fp32
    distances."""
    x = oracle.gen_gaussian(5000, 128, 50) * np.float32(1e3)
    q = oracle.gen_gaussian(20, 128, 51, row0=QROW) * np.float32(1e3)
    for precision in (2, 3):
        vals, ids = _search(ctx, x, q, 10, precision=precision)
        tids, tvals = oracle.knn(q, x, 10)
        assert_knn_parity(ids, vals, tids, tvals, _true_vals(oracle, q, x, ids, 0))


@pytest.mark.parametrize("precision", [1, 3])
def test_k_equals_database_size(ctx, oracle, precision):
    x = oracle.gen_gaussian(20, 16, 52)
    q = oracle.gen_gaussian(3, 16, 53, row0=QROW)
    vals, ids = _search(ctx, x, q, 20, precision=precision)
    tids, tvals = oracle.knn(q, x, 20)
    assert_knn_parity(ids, vals, tids, tvals, _true_vals(oracle, q, x, ids, 0))
    assert all(sorted(r.tolist()) == list(range(20)) for r in ids)
