"""Pins of the IVF / k-means oracle on the CPU (no GPU): with every list probed the IVF oracle is
the flat oracle's exact k-NN; Lloyd iterations end at the means of their own assignment; the
list layout is a stable permutation."""

import numpy as np


def test_full_probe_equals_flat_oracle(oracle):
    from oracle import ivf
    x = oracle.gen_gaussian(3000, 24, 301)
    q = oracle.gen_gaussian(17, 24, 302, row0=1 << 31)
    cent = x[:12].copy()
    rows, ids, offs = ivf.build_lists(x, cent)
    v, i = ivf.search(q, cent, rows, ids, offs, 10, 12)
    tids, tvals = oracle.knn(q, x, 10)
    assert np.array_equal(i, tids)
    np.testing.assert_allclose(v, tvals, rtol=1e-6)


def test_list_layout_is_stable_permutation(oracle):
    from oracle import ivf
    x = oracle.gen_gaussian(1000, 8, 303)
    cent = x[::100].copy()
    rows, ids, offs = ivf.build_lists(x, cent, id_base=5)
    assert offs[0] == 0 and offs[-1] == 1000
    assert np.array_equal(np.sort(ids), np.arange(5, 1005))
    a = ivf.assign(x, cent)
    for c in range(cent.shape[0]):
        seg = ids[offs[c]:offs[c + 1]] - 5
        assert np.all(np.diff(seg.astype(np.int64)) > 0)       # ascending: stable
        assert np.all(a[seg] == c)
        assert np.array_equal(rows[offs[c]:offs[c + 1]], x[seg])


def test_kmeans_fixed_point(oracle):
    from oracle import ivf
    x = oracle.gen_mixture(4000, 16, 304, 8, 0.2, False)
    c, it = ivf.kmeans(x, x[:8], 200, 1e-7)
    assert it < 200
    a = ivf.assign(x, c)
    for j in range(8):
        if np.any(a == j):
            np.testing.assert_allclose(c[j], x[a == j].astype(np.float64).mean(axis=0), rtol=1e-5, atol=1e-6)


def test_probe_padding(oracle):
    from oracle import ivf
    x = oracle.gen_gaussian(50, 4, 305)
    cent = x[:10].copy()
    rows, ids, offs = ivf.build_lists(x, cent)
    v, i = ivf.search(x[:3], cent, rows, ids, offs, 40, 1)
    for qi in range(3):
        n = int(np.sum(i[qi] != 0xFFFFFFFF))
        assert n <= 40 and np.all(np.isinf(v[qi, n:]))


def test_ivf_configuration_validation():
    """KMeansConfiguration / IVFSearchConfiguration reject what the reference rejects
    (ClusteringKernels.swift:115-130, IVFKernels.swift:28-60); no GPU needed."""
    import pytest

    import vectoraccelerate_b200 as va
    cfg = va.KMeansConfiguration(num_clusters=8, dimension=16)
    assert cfg.max_iterations == 100 and cfg.convergence_threshold == 1e-4
    for bad in (dict(num_clusters=0, dimension=16), dict(num_clusters=4, dimension=0),
                dict(num_clusters=4, dimension=16, max_iterations=0),
                dict(num_clusters=4, dimension=16, convergence_threshold=0.0)):
        with pytest.raises(va.InvalidInput):
            va.KMeansConfiguration(**bad)
    assert va.IVFSearchConfiguration(16, 4, 32).nprobe == 4
    for bad in ((0, 1, 8), (4, 0, 8), (4, 5, 8), (4, 2, 0)):
        with pytest.raises(va.InvalidInput):
            va.IVFSearchConfiguration(*bad)
