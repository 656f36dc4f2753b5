"""Host logic of AcceleratedVectorIndex (handles, deletion, compaction, metadata, the filtered
iterative fetch) with the GPU fetch replaced by a brute-force stand-in; runs on CPU."""

import numpy as np
import pytest

import vectoraccelerate_b200 as va
from vectoraccelerate_b200 import _ffi


class _Index(va.AcceleratedVectorIndex):
    """Index whose fetch is a numpy brute force (squared L2, (distance, slot) order)."""

    fetches: list

    def _fetch(self, q, fetch_k):
        self.fetches.append(fetch_k)
        d = ((q[:, None, :].astype(np.float64) - self._rows[None].astype(np.float64)) ** 2).sum(-1)
        order = np.lexsort((np.tile(np.arange(d.shape[1]), (d.shape[0], 1)), d), axis=1)[:, :fetch_k]
        return np.take_along_axis(d, order, 1).astype(np.float32), order.astype(np.uint32)


def _index(dim=4):
    idx = _Index(va.IndexConfiguration.flat(dim), context=object())
    idx.fetches = []
    return idx


def test_filtered_search_doubles_fetch_until_k_pass():
    idx = _index()
    hs = idx.insert_batch(np.arange(40, dtype=np.float32)[:, None] * np.ones((1, 4), np.float32),
                          [{"parity": str(i % 4)} for i in range(40)])
    r = idx.search(np.zeros(4, np.float32), 3, filter=lambda h, m: m["parity"] == "3")
    assert [x.id for x in r.results] == [hs[3], hs[7], hs[11]]
    assert idx.fetches == [6, 12]  # 2k, then doubled (first 6 slots hold one match)
    assert r.candidates_searched == 12


def test_filtered_search_exhausts_database():
    idx = _index()
    idx.insert_batch(np.random.default_rng(0).normal(size=(10, 4)).astype(np.float32))
    r = idx.search(np.zeros(4, np.float32), 5, filter=lambda h, m: False)
    assert r.count == 0 and r.candidates_searched == 10


def test_deletion_compaction_and_metadata():
    idx = _index()
    hs = idx.insert_batch(np.eye(4, dtype=np.float32) * np.arange(1, 5, dtype=np.float32)[:, None],
                          [{"n": str(i)} for i in range(4)])
    idx.remove(hs[0])
    assert not idx.contains(hs[0]) and idx.count == 3 and idx.allocated_slots == 4
    r = idx.search(np.zeros(4, np.float32), 2)
    assert [x.id for x in r.results] == [hs[1], hs[2]]
    assert idx.fetches[-1] == 3  # fetchK = k + deletedCount
    idx.compact()
    assert idx.allocated_slots == 3 and idx.slot(hs[1]) == 0 and idx.handle(0) == hs[1]
    assert idx.metadata(hs[2]) == {"n": "2"} and idx.metadata(hs[0]) is None
    np.testing.assert_array_equal(idx.vector(hs[3]), [0, 0, 0, 4])
    assert idx.handles_where(lambda m: m is not None and m["n"] in ("1", "3")) == [hs[1], hs[3]]
    assert idx.remove_batch([hs[0], hs[1]]) == 1
    with pytest.raises(va.InvalidInput):
        idx.remove(hs[0])
    idx.set_metadata({"n": "x"}, hs[2])
    assert idx.metadata(hs[2]) == {"n": "x"}


def test_batch_search_shapes_and_errors():
    idx = _index()
    assert idx.search(np.zeros(4, np.float32), 1).count == 0  # empty index
    idx.insert_batch(np.ones((3, 4), np.float32))
    with pytest.raises(va.InvalidInput):
        idx.search(np.zeros(3, np.float32), 1)
    with pytest.raises(va.InvalidInput):
        idx.search(np.zeros(4, np.float32), 0)
    out = idx.search_batch(np.zeros((2, 4), np.float32), 5)
    assert [r.count for r in out] == [3, 3]
    assert all(x.distance == pytest.approx(4.0) for x in out[0].results)
    assert _ffi.INVALID_ID == 0xFFFFFFFF


def test_ivf_configuration_validation():
    import vectoraccelerate_b200 as va
    c = va.IndexConfiguration.ivf(8, nlist=4, nprobe=2)
    assert c.is_ivf and c.routing_threshold == 10_000 and c.capacity == 100_000
    assert not va.IndexConfiguration.flat(8).is_ivf
    with pytest.raises(va.InvalidInput):
        va.IndexConfiguration.ivf(8, nlist=4, nprobe=5)
    with pytest.raises(va.InvalidInput):
        va.IndexConfiguration.ivf(8, nlist=4, nprobe=2, metric="cosine")
