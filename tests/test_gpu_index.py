"""AcceleratedVectorIndex through the CUDA library: filtered iterative search (including fetches
past the fused search's k limit), deletion, compaction. Needs a B200."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_index_filtered_search_matches_oracle(ctx, oracle):
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(3000, 64, 61)
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.flat(64), ctx)
    hs = idx.insert_batch(x, [{"bucket": str(i % 500)} for i in range(3000)])
    q = oracle.gen_gaussian(3, 64, 62, row0=1 << 31)
    tids, tvals = oracle.knn(q, x, 3000)
    for r in range(3):
        # one row in 500 passes: the 2k, 4k, ... fetches run past 1,024 (device top-k selection)
        got = idx.search(q[r], 4, filter=lambda h, m: m["bucket"] == "7")
        want = [int(i) for i in tids[r] if int(i) % 500 == 7][:4]
        assert [h.id.value for h in got.results] == [hs[i].value for i in want]
        np.testing.assert_allclose([h.distance for h in got.results], tvals[r][[list(tids[r]).index(i) for i in want]],
                                   rtol=1e-4)
    idx.remove_batch([hs[7], hs[507]])
    idx.compact()
    got = idx.search(q[0], 2, filter=lambda h, m: m["bucket"] == "7")
    want = [int(i) for i in tids[0] if int(i) % 500 == 7 and int(i) not in (7, 507)][:2]
    assert [h.id.value for h in got.results] == [hs[i].value for i in want]
    plain = idx.search(q[0], 5)
    want = [int(i) for i in tids[0] if int(i) not in (7, 507)][:5]
    assert [h.id.value for h in plain.results] == [hs[i].value for i in want]


def test_index_device_ingestion_matches_rebuild(ctx, oracle):
    """Inserts after the first search append on the device, compaction gathers on the device:
    results equal a fresh index over the same live rows."""
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(4000, 32, 63)
    q = oracle.gen_gaussian(5, 32, 64, row0=1 << 31)
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.flat(32), ctx)
    hs = idx.insert_batch(x[:1000])
    idx.search(q[0], 3)  # creates the device database
    hs += idx.insert_batch(x[1000:2500])
    hs += idx.insert_batch(x[2500:])
    idx.remove_batch(hs[::7])
    idx.compact()
    live = np.array([i for i in range(4000) if i % 7 != 0])
    tids, _ = oracle.knn(q, x[live], 6)
    got = idx.search_batch(q, 6)
    for r in range(5):
        assert [h.id.value for h in got[r].results] == [hs[live[i]].value for i in tids[r]]


def test_index_filtered_search_past_the_device_selection_limit(ctx, oracle):
    """A filter so selective that the doubling fetch passes 4,096 candidates: the remaining
    candidates pass the filter first and the device search orders them (no host sort)."""
    import vectoraccelerate_b200 as va
    x = oracle.gen_gaussian(30_000, 32, 71)
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.flat(32), ctx)
    hs = idx.insert_batch(x, [{"tag": i % 7919 == 3} for i in range(30_000)])
    q = oracle.gen_gaussian(2, 32, 72, row0=1 << 31)
    tids, tvals = oracle.knn(q, x, 30_000)
    for r in range(2):
        got = idx.search(q[r], 3, filter=lambda h, m: m["tag"])
        want = [int(i) for i in tids[r] if int(i) % 7919 == 3][:3]
        assert [h.id.value for h in got.results] == [hs[i].value for i in want]
        np.testing.assert_allclose([h.distance for h in got.results],
                                   tvals[r][[list(tids[r]).index(i) for i in want]], rtol=1e-4)
