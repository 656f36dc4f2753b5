"""AcceleratedVectorIndex in IVF mode (IndexConfiguration.ivf): routing, training, deletion and
filtering against the flat index and the IVF oracle. Needs a B200."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

QROW = 1 << 31


def _ids(res):
    return [r.id.value for r in res.results]


def test_untrained_and_below_threshold_route_to_flat(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(3000, 32, 501)
    q = oracle.gen_gaussian(5, 32, 502, row0=QROW)
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.ivf(32, nlist=16, nprobe=2, routing_threshold=0,
                                                              min_training_vectors=10**9), context=ctx)
    hs = idx.insert_batch(x)
    assert idx.is_ivf and not idx.is_trained
    res = idx.search_batch(q, 10)
    tids, _ = oracle.knn(q, x, 10)
    for r in range(5):
        assert _ids(res[r]) == [hs[i].value for i in tids[r]] and res[r].is_exhaustive
    idx.train()
    assert idx.is_trained
    # above the routing threshold (0 = always): IVF, approximate
    assert not idx.search_batch(q, 10)[0].is_exhaustive
    idx2 = va.AcceleratedVectorIndex(va.IndexConfiguration.ivf(32, nlist=16, nprobe=2, routing_threshold=5000),
                                     context=ctx)
    idx2.insert_batch(x)
    idx2.train()
    assert idx2.search_batch(q, 10)[0].is_exhaustive     # 3000 live < 5000: flat


def test_auto_training_and_full_probe_equals_flat(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_mixture(12000, 48, 503, 32, 0.4, False)
    q = oracle.gen_mixture(20, 48, 503, 32, 0.4, False, row0=QROW)
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.ivf(48, nlist=24, nprobe=24, routing_threshold=0,
                                                              min_training_vectors=8000), context=ctx)
    hs = idx.insert_batch(x[:7000])
    assert not idx.is_trained
    hs += idx.insert_batch(x[7000:])                       # crosses min_training_vectors
    assert idx.is_trained
    res = idx.search_batch(q, 10)                          # every list probed: the exact answer
    tids, tvals = oracle.knn(q, x, 10)
    for r in range(20):
        assert _ids(res[r]) == [hs[i].value for i in tids[r]]
        np.testing.assert_allclose([t.distance for t in res[r].results], tvals[r], rtol=1e-5, atol=1e-6)


def test_ivf_index_matches_oracle_with_deletions(ctx, oracle):
    import vectoraccelerate_b200 as va
    from oracle import ivf as O
    x = oracle.gen_mixture(20000, 64, 505, 40, 0.4, False)
    q = oracle.gen_mixture(15, 64, 505, 40, 0.4, False, row0=QROW)
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.ivf(64, nlist=32, nprobe=6, routing_threshold=0,
                                                              min_training_vectors=10**9), context=ctx)
    hs = idx.insert_batch(x)
    idx.train()
    dead = set(range(0, 20000, 7))
    idx.remove_batch([hs[i] for i in dead])
    res = idx.search_batch(q, 10)
    cent = idx._centroids
    rows, ids, offs = O.build_lists(x, cent)
    tv, ti = O.search(q, cent, rows, ids, offs, 10 + len(dead) if 10 + len(dead) <= 128 else 128, 6)
    for r in range(15):
        want = [int(i) for i in ti[r] if i != 0xFFFFFFFF and int(i) not in dead][:10]
        got = _ids(res[r])
        assert got == [hs[i].value for i in want] or np.allclose(
            sorted(t.distance for t in res[r].results),
            sorted(float(np.sum((x[i].astype(np.float64) - q[r]) ** 2)) for i in want), rtol=1e-5)
    # compaction keeps the trained centroids and rebuilds the lists
    idx.compact()
    res2 = idx.search_batch(q, 10)
    assert [_ids(a) for a in res2] == [_ids(b) for b in res]


def test_ivf_filtered_single_query(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(5000, 16, 507)
    q = oracle.gen_gaussian(1, 16, 508, row0=QROW)[0]
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.ivf(16, nlist=8, nprobe=8, routing_threshold=0,
                                                              min_training_vectors=10**9), context=ctx)
    hs = idx.insert_batch(x, metadata=[{"p": str(i % 3)} for i in range(5000)])
    idx.train()
    res = idx.search(q, 5, filter=lambda h, m: m["p"] != "0")   # over-fetch 15, keep what passes
    tids, _ = oracle.knn(q[None, :], x, 15)
    want = [int(i) for i in tids[0] if i % 3 != 0][:5]
    assert len(want) == 5 and res.count == 5 and not res.is_exhaustive
    assert _ids(res) == [hs[i].value for i in want]
