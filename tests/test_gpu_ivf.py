"""IVF search and k-means on the device (va_ivf_*) against the numpy IVF oracle. Needs a B200."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

QROW = 1 << 31


def _true_vals(q, x_by_id, ids):
    out = np.full(ids.shape, np.inf, np.float32)
    for r in range(ids.shape[0]):
        for j in range(ids.shape[1]):
            if ids[r, j] != 0xFFFFFFFF:
                d = x_by_id[ids[r, j]].astype(np.float64) - q[r].astype(np.float64)
                out[r, j] = np.float32(np.dot(d, d))
    return out


# k <= 42 takes the tensor-core list scan with bf16 keys, 43 <= k <= 103 with tf32 keys (both an
# exact rerank of a candidate pool), larger k the exact fp64 scan; all must give the oracle's
# answer.
@pytest.mark.parametrize("dim,nlist,nprobe,k", [(64, 32, 1, 10), (64, 32, 4, 10), (96, 16, 16, 100),
                                                (128, 64, 8, 128), (7, 10, 3, 5), (64, 32, 8, 42),
                                                (48, 20, 5, 43), (200, 40, 40, 1), (100, 24, 6, 103),
                                                (64, 32, 8, 104), (128, 32, 4, 60)])
def test_ivf_search_parity(ctx, oracle, dim, nlist, nprobe, k):
    import vectoraccelerate_b200 as va
    from oracle import ivf as O
    from conftest import assert_knn_parity
    x = oracle.gen_mixture(20000, dim, 400 + dim, 48, 0.4, False)
    q = oracle.gen_mixture(70, dim, 400 + dim, 48, 0.4, False, row0=QROW)
    cent = x[::20000 // nlist][:nlist].copy()
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(nlist, nprobe, dim))
    st = pipe.build(x, cent)
    try:
        rows, ids, offs = O.build_lists(x, cent)
        assert np.array_equal(st.list_sizes, np.diff(offs))
        res = pipe.search(q, st, k)
        tv, ti = O.search(q, cent, rows, ids, offs, k, nprobe)
        assert_knn_parity(res.indices, res.distances, ti, tv, _true_vals(q, x, res.indices))
    finally:
        st.close()


def test_full_probe_equals_exact(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(8000, 48, 410)
    q = oracle.gen_gaussian(25, 48, 411, row0=QROW)
    cent = x[:20].copy()
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(20, 20, 48))
    st = pipe.build(x, cent, id_base=1000)
    try:
        res = pipe.search(q, st, 10)
        tids, tvals = oracle.knn(q, x, 10)
        assert np.array_equal(res.indices, tids + 1000)
        np.testing.assert_allclose(res.distances, tvals, rtol=1e-5, atol=1e-6)
    finally:
        st.close()


def test_prepare_from_host_lists(ctx, oracle):
    import vectoraccelerate_b200 as va
    from oracle import ivf as O
    x = oracle.gen_gaussian(3000, 32, 412)
    q = oracle.gen_gaussian(9, 32, 413, row0=QROW)
    cent = x[:8].copy()
    a = O.assign(x, cent)
    lists = [x[a == c] for c in range(8)]
    lists[3] = np.zeros((0, 32), np.float32)              # an empty list
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(8, 3, 32))
    st = pipe.prepare_index_structure(cent, lists)
    try:
        rows = np.concatenate(lists)
        offs = np.concatenate([[0], np.cumsum([len(l) for l in lists])]).astype(np.int64)
        flat = np.arange(rows.shape[0], dtype=np.uint32)   # the reference's ids: flat positions
        assert st.total_vectors == rows.shape[0] and st.list_count(3) == 0
        res = pipe.search(q, st, 20)
        tv, ti = O.search(q, cent, rows, flat, offs, 20, 3)
        from conftest import assert_knn_parity
        assert_knn_parity(res.indices, res.distances, ti, tv, _true_vals(q, rows, res.indices))
    finally:
        st.close()


def test_padding_when_lists_are_short(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(60, 16, 414)
    cent = x[:12].copy()
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(12, 1, 16))
    st = pipe.build(x, cent)
    try:
        res = pipe.search(x[:12], st, 64)
        for qi in range(12):
            # x[qi] is centroid qi, so its one probe is list qi: every row of it, then padding.
            got = int(np.sum(res.indices[qi] != 0xFFFFFFFF))
            assert got == min(64, st.list_count(qi))
            assert np.all(np.isinf(res.distances[qi, got:])) and np.all(res.indices[qi, got:] == 0xFFFFFFFF)
            assert res.indices[qi, 0] == qi and res.distances[qi, 0] == 0.0
    finally:
        st.close()


def test_ivf_invalid_arguments(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(500, 16, 415)
    with pytest.raises(va.InvalidInput):
        va.IVFSearchConfiguration(4, 5, 16)
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(4, 2, 16))
    st = pipe.build(x, x[:4].copy())
    try:
        with pytest.raises(va.InvalidInput):
            pipe.search(x[:2], st, 129)
        with pytest.raises(va.InvalidInput):
            pipe.search(x[:2, :8], st, 5)
    finally:
        st.close()


def test_kmeans_parity_from_given_centroids(ctx, oracle):
    import vectoraccelerate_b200 as va
    from oracle import ivf as O
    x = oracle.gen_mixture(30000, 32, 420, 16, 0.3, False)
    init = x[:16].copy()
    cfg = va.KMeansConfiguration(num_clusters=16, dimension=32, max_iterations=12, convergence_threshold=1e-4)
    r = va.KMeansPipeline(ctx, cfg).fit(x, initial_centroids=init)
    c, it = O.kmeans(x, init, 12, 1e-4)
    assert r.iterations == it
    np.testing.assert_allclose(r.centroids, c, rtol=1e-5, atol=1e-6)
    assert np.array_equal(r.assignments, O.assign(x, r.centroids))


def test_kmeans_seeded_is_deterministic_and_converges(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(20000, 24, 421, 10, 0.2, False)
    cfg = va.KMeansConfiguration(num_clusters=10, dimension=24, max_iterations=100, convergence_threshold=1e-5,
                                 seed=7)
    a = va.KMeansPipeline(ctx, cfg).fit(x)
    b = va.KMeansPipeline(ctx, cfg).fit(x)
    assert np.array_equal(a.centroids, b.centroids) or np.allclose(a.centroids, b.centroids, rtol=1e-6)
    assert a.converged and a.iterations < 100
    for j in range(10):
        m = a.assignments == j
        if m.any():
            np.testing.assert_allclose(a.centroids[j], x[m].astype(np.float64).mean(axis=0), rtol=1e-4, atol=1e-5)


def test_ivf_many_lists_coarse_tf32(ctx, oracle):
    """More than 16,384 lists: the coarse quantizer takes the tensor-core (TF32) route. With the
    rows themselves as centroids every list holds its own row, so probing the 8 nearest lists
    returns the exact 8 nearest rows."""
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(20000, 32, 430)
    q = oracle.gen_gaussian(12, 32, 431, row0=QROW)
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(20000, 8, 32))
    st = pipe.build(x, x)
    try:
        assert st.total_vectors == 20000 and int(st.list_sizes.max()) == 1
        res = pipe.search(q, st, 8)
        tids, tvals = oracle.knn(q, x, 8)
        assert np.array_equal(res.indices, tids)
        np.testing.assert_allclose(res.distances, tvals, rtol=1e-5, atol=1e-6)
    finally:
        st.close()


def test_kmeanspp_seeds(ctx, oracle):
    """k-means++ seeds (max_iters = 0): distinct rows of the data, the same for the same seed, and
    on well-separated clusters one seed per cluster (D^2 sampling)."""
    import ctypes

    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi
    rng = np.random.default_rng(5)
    centers = rng.normal(size=(8, 16)).astype(np.float32) * 20
    lab = np.repeat(np.arange(8), 500)
    x = (centers[lab] + rng.normal(size=(4000, 16)).astype(np.float32) * 0.05).astype(np.float32)

    def seeds(seed):
        dx = ctx.get_buffer_for(x)
        dc = ctx.get_buffer(8 * 16 * 4, np.float32, (8, 16))
        it = ctypes.c_int(-1)
        _ffi.call("va_ivf_train", ctx.handle, dx.ptr, 4000, 16, 8, 0, ctypes.c_float(1e-3), seed,
                  _ffi.IVF_INIT_KMEANSPP, dc.ptr, ctypes.byref(it))
        assert it.value == 0
        return dc.download()

    a, b, c = seeds(11), seeds(11), seeds(12)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    rows = [int(np.where((x == s).all(axis=1))[0][0]) for s in a]   # every seed is a row
    assert len(set(rows)) == 8 and sorted(set(lab[rows])) == list(range(8))
    km = va.KMeansPipeline(ctx, va.KMeansConfiguration(num_clusters=8, dimension=16, max_iterations=20)).fit(x)
    assert km.converged and len(set(km.assignments[lab == 0])) == 1


@pytest.mark.parametrize("k", [10, 60])
def test_ivf_certificate_rescans_near_duplicates(ctx, oracle, k):
    """Runs of near-duplicate rows inside a list defeat the list scan's certificate: those queries
    are rescanned exactly and the result still equals the oracle's (exact within the probes)."""
    import vectoraccelerate_b200 as va
    from oracle import ivf as O
    from conftest import assert_knn_parity
    rng = np.random.default_rng(5 + k)
    x = rng.standard_normal((20_000, 64)).astype(np.float32)
    q = rng.standard_normal((12, 64)).astype(np.float32)
    runs = [q[i] + 0.3 * rng.standard_normal(64).astype(np.float32) for i in range(4)]
    dup = np.concatenate([p[None, :] + 1e-3 * rng.standard_normal((300, 64)).astype(np.float32) for p in runs])
    x = np.concatenate([x, dup]).astype(np.float32)
    cent = x[::1000][:16].copy()
    pipe = va.IVFSearchPipeline(ctx, va.IVFSearchConfiguration(16, 4, 64))
    st = pipe.build(x, cent)
    try:
        rows, ids, offs = O.build_lists(x, cent)
        res = pipe.search(q, st, k)
        assert ctx.last_search_stats()[0] >= 1
        tv, ti = O.search(q, cent, rows, ids, offs, k, 4)
        assert_knn_parity(res.indices, res.distances, ti, tv, _true_vals(q, x, res.indices))
    finally:
        st.close()
