"""GPU parity of candidate pools wider than the filter's 128-entry lists: int8 search with 1,000
rerank candidates (the benchmark's int8 configuration, smaller database) and float searches whose
pool exceeds 128, including data that forces the exact fallback (long runs of duplicate rows put
more than 128 of a query's pool into one row split). Needs a B200."""

import numpy as np
import pytest

from conftest import assert_knn_parity

pytestmark = pytest.mark.gpu

QROW = 1 << 31


def _true(q, x, ids, metric=0):
    valid = ids != 0xFFFFFFFF
    safe = np.where(valid, ids, 0).astype(np.int64)
    qq = q[:, None, :].astype(np.float64)
    xx = x[safe].astype(np.float64)
    if metric == 0:
        d = ((qq - xx) ** 2).sum(-1)
    elif metric == 2:
        d = (qq * xx).sum(-1)
    else:
        num = (qq * xx).sum(-1)
        den = np.sqrt((qq ** 2).sum(-1)) * np.sqrt((xx ** 2).sum(-1))
        d = 1.0 - np.clip(np.where(den > 0, num / np.where(den > 0, den, 1), 0.0), -1, 1)
    return np.where(valid, d, np.nan).astype(np.float32)


def _int8_oracle(oracle, x, q, cand, k):
    mins, scales = oracle.sq_perdim_params(x)
    xc = oracle.sq_perdim_quantize(x, mins, scales)
    qc = oracle.sq_perdim_quantize(q, mins, scales)
    oids, ovals, _, _ = oracle.int8_knn(qc, q, xc, x, cand, k)
    return oids, ovals


@pytest.mark.parametrize("n,nq,k,cand", [(50_000, 300, 100, 1000), (20_000, 129, 10, 200), (3000, 64, 5, 4096)])
def test_int8_wide_pool(ctx, oracle, n, nq, k, cand):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(n, 768, 11, 256, 0.3, False)
    q = oracle.gen_mixture(nq, 768, 11, 256, 0.3, False, row0=QROW)
    oids, ovals = _int8_oracle(oracle, x, q, cand, k)
    db = va.Int8Database(ctx, x)
    try:
        vals, ids = db.search(q, k, cand)
    finally:
        db.close()
    assert_knn_parity(ids, vals, oids, ovals, _true(q, x, ids))


def _clustered(oracle, reps, dim, seed):
    """Rows in long runs of duplicates: base row i repeated `reps` times contiguously."""
    base = oracle.gen_gaussian(64, dim, seed)
    return base, np.repeat(base, reps, axis=0)


def test_int8_wide_pool_fallback(ctx, oracle):
    """Queries equal to a base row have their 400 duplicates (distance 0) inside one or two row
    splits, so their pool cannot be proven from 128-entry lists and takes the exact scan; other
    queries (fresh Gaussian rows) mostly pass the proof. Results must match either way."""
    import vectoraccelerate_b200 as va
    base, x = _clustered(oracle, 400, 256, 21)
    q = np.concatenate([base[:20], oracle.gen_gaussian(44, 256, 21, row0=QROW)])
    oids, ovals = _int8_oracle(oracle, x, q, 1000, 50)
    db = va.Int8Database(ctx, x)
    try:
        vals, ids = db.search(q, 50, 1000)
    finally:
        db.close()
    assert_knn_parity(ids, vals, oids, ovals, _true(q, x, ids))


@pytest.mark.parametrize("metric,k,rerank", [(0, 200, 0), (0, 10, 20), (1, 150, 0), (2, 300, 2)])
def test_float_wide_pool(ctx, oracle, metric, k, rerank):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(30_000, 768, 13, 128, 0.3, metric == 1)
    q = oracle.gen_mixture(257, 768, 13, 128, 0.3, metric == 1, row0=QROW)
    tids, tvals = oracle.knn(q, x, k, metric=metric)
    db = va.Database(ctx, x)
    try:
        vals, ids = va.knn_search_host(ctx, db, q, k, metric, va.PREC_AUTO, rerank)
    finally:
        db.close()
    assert_knn_parity(ids, vals, tids, tvals, _true(q, x, ids, metric), larger_is_better=metric == 2)


def test_float_wide_pool_fallback(ctx, oracle):
    import vectoraccelerate_b200 as va
    base, x = _clustered(oracle, 400, 768, 23)
    q = np.concatenate([base[:16], oracle.gen_gaussian(48, 768, 23, row0=QROW)])
    tids, tvals = oracle.knn(q, x, 200, metric=0)
    db = va.Database(ctx, x)
    try:
        vals, ids = va.knn_search_host(ctx, db, q, 200, 0, va.PREC_BF16, 0)
    finally:
        db.close()
    assert_knn_parity(ids, vals, tids, tvals, _true(q, x, ids))
