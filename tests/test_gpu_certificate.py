"""The exactness certificate of the reduced-precision search, on a B200.

The tensor-core filter ranks rows by bf16 (or tf32) keys; the merge reranks its candidate pool
exactly and certifies per query that no row outside the pool can enter the top k (a rigorous
bound of the keys' rounding error against the gap between the k-th exact distance and the pool's
last key). Runs of near-duplicate rows closer together than that bound defeat the certificate on
purpose: those queries must take the second tensor-core pass (wider pool) or the exact route, and
the results must still equal the oracle's (CPUTopK.swift:62-79: exact sum((q - x)^2) order).
When more than 1/32 of a batch fails, the second pass widens the pool to at least 512 and the
database keeps it (dense neighbourhoods); the tests of the narrow fallbacks use batches where the
few failing queries stay under that share."""

import numpy as np
import pytest

from test_gpu_parity import _check

pytestmark = pytest.mark.gpu


def _near_duplicate_db(n, d, dup, seed, spread=1e-3, normalize=False, nq=64):
    """n random rows plus, for each of the first 4 of `nq` queries, `dup` rows within `spread` of
    one point near that query (the query's top k lie inside the run)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, d)).astype(np.float32)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    runs = []
    for i in range(4):
        p = q[i] + 0.5 * rng.standard_normal(d).astype(np.float32)
        runs.append(p[None, :] + spread * rng.standard_normal((dup, d)).astype(np.float32))
    x = np.concatenate([x[: n // 2]] + runs + [x[n // 2:]]).astype(np.float32)
    if normalize:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        q /= np.linalg.norm(q, axis=1, keepdims=True)
    return x, q


def _search(ctx, x, q, k, metric=0, precision=0, rerank=0, dtype=0):
    import vectoraccelerate_b200 as va
    db = va.Database(ctx, x, dtype=dtype)
    try:
        vals, ids = va.knn_search_host(ctx, db, q, k, metric, precision, rerank)
        return vals, ids, ctx.last_search_stats()
    finally:
        db.close()


@pytest.mark.parametrize("metric", [0, 1, 2])
@pytest.mark.parametrize("precision", [2, 3])
def test_runs_beyond_every_pool_take_the_exact_route(ctx, oracle, metric, precision):
    # 300 near-duplicates: neither the first pool (32) nor the second (64) separates them. Four
    # failing queries of 200 (under 1/32 of the batch) keep the second pass at the next list size.
    x, q = _near_duplicate_db(20_000, 128, 300, seed=11 + metric, normalize=metric == 1, nq=200)
    vals, ids, (unc, exact) = _search(ctx, x, q, 10, metric=metric, precision=precision)
    assert unc >= 4 and exact >= 4, (unc, exact)
    _check(oracle, q, x, 10, metric, vals, ids)


def test_runs_inside_the_second_pool_are_certified_there(ctx, oracle):
    # 50 near-duplicates: the first pool (32) cannot separate them, the second (64) holds them all.
    x, q = _near_duplicate_db(20_000, 128, 50, seed=5, nq=200)
    vals, ids, (unc, exact) = _search(ctx, x, q, 10, precision=3)
    assert unc >= 4 and exact == 0, (unc, exact)
    _check(oracle, q, x, 10, 0, vals, ids)


def test_bf16_rows_exact_route(ctx, oracle):
    # bf16 rows: the exact route reads the bf16 rows widened exactly
    x, q = _near_duplicate_db(10_000, 128, 300, seed=3, normalize=True, nq=200)
    xb = oracle.f32_to_bf16(x)
    vals, ids, (unc, exact) = _search(ctx, xb, q, 10, metric=2, precision=3, dtype=1)
    assert exact >= 4
    _check(oracle, q, xb, 10, 2, vals, ids, db_bf16=True)


def test_random_data_certifies_nearly_all(ctx, oracle):
    # No near-duplicates: the first pass certifies (almost) every query and results are exact.
    rng = np.random.default_rng(2)
    x = rng.standard_normal((50_000, 256)).astype(np.float32)
    q = rng.standard_normal((300, 256)).astype(np.float32)
    vals, ids, (unc, exact) = _search(ctx, x, q, 10)
    assert unc <= 30 and exact == 0, (unc, exact)
    _check(oracle, q, x, 10, 0, vals, ids)


def test_wide_pool_certificate(ctx, oracle):
    # k = 60 under AUTO: a 180-candidate pool from 64/128-entry lists, proven and certified
    x, q = _near_duplicate_db(30_000, 96, 400, seed=9)
    vals, ids, (unc, exact) = _search(ctx, x, q, 60)
    assert unc >= 4
    _check(oracle, q, x, 60, 0, vals, ids)


def test_dense_neighbourhoods_widen_the_pool_and_are_remembered(ctx, oracle):
    # Every query sits next to its own run of 200 near-duplicates: the whole batch fails the first
    # pool (32), the second pass takes a pool of 512 (more than the run), and the database keeps
    # that pool for its next searches of the metric, which then certify in their first pass.
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(21)
    q = rng.standard_normal((80, 96)).astype(np.float32)
    runs = [q[i] + 0.5 * rng.standard_normal(96).astype(np.float32) for i in range(80)]
    x = np.concatenate([rng.standard_normal((10_000, 96)).astype(np.float32)] +
                       [p[None, :] + 1e-3 * rng.standard_normal((200, 96)).astype(np.float32) for p in runs])
    x = np.ascontiguousarray(x[rng.permutation(len(x))])  # a run's rows spread over the row splits
    db = va.Database(ctx, x)
    try:
        vals, ids = va.knn_search_host(ctx, db, q, 10, 0, va.PREC_BF16)
        unc, exact = ctx.last_search_stats()
        assert unc == 80 and exact == 0, (unc, exact)
        _check(oracle, q, x, 10, 0, vals, ids)
        vals, ids = va.knn_search_host(ctx, db, q, 10, 0, va.PREC_BF16)
        assert ctx.last_search_stats() == (0, 0)
        _check(oracle, q, x, 10, 0, vals, ids)
    finally:
        db.close()


@pytest.mark.parametrize("metric", [0, 2])
def test_merge_extension_certifies_without_a_second_pass(ctx, oracle, metric):
    # 40 near-duplicates per run (more than the pool of 32, closer together than the key error)
    # spread over the row splits: the pool test fails for those queries, but every split's list
    # ends far above them, so the merge reranks the whole run and certifies in the first pass.
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(41 + metric)
    q = rng.standard_normal((200, 128)).astype(np.float32)
    runs = [q[i] + 0.5 * rng.standard_normal(128).astype(np.float32) for i in range(4)]
    x = np.concatenate([rng.standard_normal((30_000, 128)).astype(np.float32)] +
                       [p[None, :] + 1e-3 * rng.standard_normal((40, 128)).astype(np.float32) for p in runs])
    x = np.ascontiguousarray(x[rng.permutation(len(x))])
    db = va.Database(ctx, x)
    try:
        vals, ids = va.knn_search_host(ctx, db, q, 10, metric, va.PREC_BF16)
        assert ctx.last_search_stats() == (0, 0)
        _check(oracle, q, x, 10, metric, vals, ids)
    finally:
        db.close()
