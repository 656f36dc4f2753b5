"""MetalComputeProvider through the CUDA library against the oracle. Needs a B200."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric,om", [("euclidean", 0), ("cosine", 1), ("dotProduct", 2)])
def test_provider_find_nearest_and_batch_distance(ctx, oracle, metric, om):
    import vectoraccelerate_b200 as va
    p = va.MetalComputeProvider(ctx)
    x = oracle.gen_gaussian(2500, 48, 71)
    q = oracle.gen_gaussian(4, 48, 72, row0=1 << 31)
    tids, tvals = oracle.knn(q, x, 12, metric=om)
    got = p.find_nearest_batch(q, x, 12, metric)
    for r in range(4):
        assert [i for i, _ in got[r]] == tids[r].tolist()
        want = np.sqrt(tvals[r]) if metric == "euclidean" else tvals[r]
        np.testing.assert_allclose([d for _, d in got[r]], want, rtol=1e-4, atol=1e-5)
    one = p.find_nearest(q[0], x, 3, metric)
    assert [i for i, _ in one] == tids[0][:3].tolist()
    d = p.batch_distance(q[1], x, metric)
    full = oracle.matrix(q[1:2], x, om, flag=metric in ("euclidean", "cosine"))[0]
    np.testing.assert_allclose(d, full, rtol=2e-4, atol=1e-4)


def test_provider_edges(ctx):
    import vectoraccelerate_b200 as va
    p = va.MetalComputeProvider(ctx)
    assert p.find_nearest(np.zeros(4, np.float32), np.zeros((0, 4), np.float32), 3, "euclidean") == []
    assert p.batch_distance(np.zeros(4, np.float32), np.zeros((0, 4), np.float32), "cosine").size == 0
    with pytest.raises(va.InvalidInput):
        p.batch_distance(np.zeros(4, np.float32), np.zeros((2, 5), np.float32), "euclidean")
    with pytest.raises(va.Unsupported):
        p.find_nearest(np.zeros(4, np.float32), np.ones((2, 4), np.float32), 1, "manhattan")
    res = p.find_nearest(np.zeros(2, np.float32), np.array([[3, 4], [1, 0]], np.float32), 5, "euclidean")
    assert res == [(1, 1.0), (0, 5.0)]  # k clipped to the candidate count; sqrt distances
