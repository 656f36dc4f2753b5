"""AcceleratedVectorIndex: the flat-index caller of the fused search.

Mirrors Index/AcceleratedVectorIndex.swift for the flat path: ``insert`` returns a stable
``VectorHandle`` (with optional string metadata, :481-560); ``remove`` marks a slot deleted (lazy
deletion, Index/Internal/DeletionMask.swift; :771-832); ``compact`` drops deleted slots and remaps
handles (:834-893); ``search(query:k:filter:)`` (:895-945) runs the GPU search with
``fetchK = min(k + deletedCount, allocatedSlots)`` (:1146-1147), drops deleted slots and maps
slot -> handle (:1162-1177); a filter runs the reference's iterative fetch (start at 2k, double
until k results pass or every slot was seen, :1188-1265); ``search(queries:k:filter:)`` (:947-1000)
batches unfiltered queries in one GPU call. Distances are squared L2 (the reference's index is
euclidean-only, :305-315); cosine and inner product are accepted here as an extension.

Rows live in a resident device database created on the first search and then kept in step on
the device: inserts append to it (va_db_append, geometric growth) and compaction gathers its kept
rows (va_db_compact), as GPUVectorStorage writes and compacts its buffer. A host copy of the rows
serves ``vector(for:)`` and the exhaustive tail of a filtered search.

IVF indexes (``IndexConfiguration.ivf``, IndexConfiguration.swift:274-290,347-370) follow the
reference's routing: until trained, and while fewer vectors than ``routing_threshold`` are live,
searches are flat; ``train()`` (:396-446) runs k-means over the live vectors (25 iterations,
movement threshold 1e-3, as IVFStructure.swift:218-222) and inserts train automatically once
``min_training_vectors`` (default max(10 nlist, 1000), IVFStructure.swift:187) are staged
(:529-545). A trained index searches its lists (searchIVF / searchIVFBatch, :1378-1470): the
lists are rebuilt on the device from the resident rows after any change, slots are the ids, and
deleted slots are skipped after an over-fetch of k + deleted (at most 128); a filtered single-query
search over-fetches 3k and filters (:1397-1420). k above 128 is served by the flat search.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np

from . import _ffi
from .context import GPUContext
from .errors import IndexError as VAIndexError
from .kernels import Database, knn_search_host

_METRICS = {"euclidean": _ffi.METRIC_L2SQ, "cosine": _ffi.METRIC_COSINE, "dot": _ffi.METRIC_IP}

VectorMetadata = dict  # [String: String] (AcceleratedVectorIndex.swift:22)


@dataclass(frozen=True)
class IndexConfiguration:
    """IndexConfiguration (Index/Types/IndexConfiguration.swift:230-370): ``flat(...)`` and
    ``ivf(...)``. index_type is ("flat",) or ("ivf", nlist, nprobe, min_training_vectors)."""

    dimension: int
    metric: str = "euclidean"
    capacity: int = 1024
    index_type: tuple = ("flat",)
    routing_threshold: int = 0

    @staticmethod
    def flat(dimension: int, metric: str = "euclidean", capacity: int = 1024) -> "IndexConfiguration":
        return IndexConfiguration(dimension, metric, capacity)

    @staticmethod
    def ivf(dimension: int, nlist: int, nprobe: int, metric: str = "euclidean", capacity: int = 100_000,
            routing_threshold: int = 10_000, min_training_vectors: Optional[int] = None) -> "IndexConfiguration":
        if nlist <= 0 or not 1 <= nprobe <= nlist:
            raise VAIndexError(f"IVF needs nlist > 0 and 1 <= nprobe <= nlist, got {nlist} / {nprobe}")
        if metric != "euclidean":
            raise VAIndexError("the IVF index is euclidean (squared L2) only")
        return IndexConfiguration(dimension, metric, capacity, ("ivf", nlist, nprobe, min_training_vectors),
                                  routing_threshold)

    @property
    def is_ivf(self) -> bool:
        return self.index_type[0] == "ivf"


@dataclass(frozen=True)
class VectorHandle:
    value: int


@dataclass(frozen=True)
class IndexSearchResult:
    id: VectorHandle
    distance: float


@dataclass
class SearchResults:
    """SearchResults<VectorHandle> (Index/Types/SearchResult.swift): results plus the number of
    candidates examined and whether the search was exhaustive."""

    results: list
    candidates_searched: int = 0
    is_exhaustive: bool = True

    @property
    def count(self) -> int:
        return len(self.results)


Filter = Callable[[VectorHandle, Optional[VectorMetadata]], bool]


class AcceleratedVectorIndex:
    def __init__(self, configuration: IndexConfiguration, context: GPUContext | None = None,
                 precision: int = _ffi.PREC_AUTO):
        if configuration.dimension <= 0:
            raise VAIndexError(f"dimension must be positive, got {configuration.dimension}")
        if configuration.metric not in _METRICS:
            raise VAIndexError(f"unsupported metric {configuration.metric!r}")
        self.configuration = configuration
        self.context = context or GPUContext()
        self.precision = precision
        # Host copy of the rows in preallocated capacity that grows geometrically (as the device
        # storage does, GPUVectorStorage.swift:75-260), so inserts are amortized O(rows written).
        self._row_buf = np.zeros((0, configuration.dimension), np.float32)
        self._del_buf = np.zeros(0, bool)
        self._n = 0
        self._slot_handle: list[int] = []          # slot -> handle value
        self._handle_slot: dict[int, int] = {}     # live handle value -> slot
        self._metadata: dict[int, VectorMetadata] = {}
        self._next_handle = 0
        self._db: Database | None = None
        # IVF state: trained centroids, the device lists (rebuilt after any change), auto-training
        self._centroids: np.ndarray | None = None
        self._ivf = None
        self._ivf_dirty = True
        self._auto_train = True

    # ------------------------------------------------------------------------- storage
    @property
    def _rows(self) -> np.ndarray:
        return self._row_buf[:self._n]

    @property
    def _deleted(self) -> np.ndarray:
        return self._del_buf[:self._n]

    def _append_rows(self, v: np.ndarray) -> int:
        """Write rows after the last slot (capacity at least doubles when full); returns the first slot."""
        slot0, need = self._n, self._n + v.shape[0]
        if need > self._row_buf.shape[0]:
            cap = max(need, 2 * self._row_buf.shape[0], 256)
            rows = np.zeros((cap, self.configuration.dimension), np.float32)
            rows[:slot0] = self._row_buf[:slot0]
            dele = np.zeros(cap, bool)
            dele[:slot0] = self._del_buf[:slot0]
            self._row_buf, self._del_buf = rows, dele
        self._row_buf[slot0:need] = v
        self._del_buf[slot0:need] = False
        self._n = need
        return slot0

    # ------------------------------------------------------------------------- mutation
    def insert(self, vector, metadata: Optional[VectorMetadata] = None) -> VectorHandle:
        return self.insert_batch([vector], None if metadata is None else [metadata])[0]

    def insert_batch(self, vectors, metadata: Optional[list] = None) -> list[VectorHandle]:
        v = np.ascontiguousarray(vectors, np.float32)
        if v.ndim == 1:
            v = v[None, :]
        if v.shape[1] != self.configuration.dimension:
            raise VAIndexError(f"dimension mismatch: expected {self.configuration.dimension}, got {v.shape[1]}")
        if metadata is not None and len(metadata) != v.shape[0]:
            raise VAIndexError(f"metadata count {len(metadata)} != vector count {v.shape[0]}")
        slot0 = self._append_rows(v)
        handles = []
        for i in range(v.shape[0]):
            h = self._next_handle
            self._next_handle += 1
            self._slot_handle.append(h)
            self._handle_slot[h] = slot0 + i
            if metadata is not None and metadata[i] is not None:
                self._metadata[h] = dict(metadata[i])
            handles.append(VectorHandle(h))
        if self._db is not None:
            self._db.append(v)
        self._ivf_dirty = True
        cfg = self.configuration
        if cfg.is_ivf and self._centroids is None and self._auto_train:
            min_train = cfg.index_type[3] or max(10 * cfg.index_type[1], 1000)
            if self.count >= min_train:
                self.train()
        return handles

    def remove(self, handle: VectorHandle) -> None:
        slot = self._handle_slot.pop(handle.value, None)
        if slot is None:
            raise VAIndexError(f"unknown handle {handle.value}")
        self._deleted[slot] = True
        self._metadata.pop(handle.value, None)
        self._ivf_dirty = True

    def remove_batch(self, handles) -> int:
        """remove(_ handles:) (:800-832): removes the live ones, returns how many."""
        n = 0
        for h in handles:
            if h.value in self._handle_slot:
                self.remove(h)
                n += 1
        return n

    def compact(self) -> None:
        """Drop deleted slots; live handles keep their values and move to new slots."""
        if not self._deleted.any():
            return
        keep = ~self._deleted
        if self._db is not None:
            if keep.any():
                self._db.compact(keep)
            else:
                self._db.close()
                self._db = None
        self._ivf_dirty = True
        kept = np.ascontiguousarray(self._rows[keep])
        self._n = 0
        self._append_rows(kept)
        self._slot_handle = [h for h, k in zip(self._slot_handle, keep) if k]
        self._handle_slot = {h: s for s, h in enumerate(self._slot_handle)}

    def set_metadata(self, metadata: Optional[VectorMetadata], handle: VectorHandle) -> None:
        if handle.value not in self._handle_slot:
            raise VAIndexError(f"unknown handle {handle.value}")
        if metadata is None:
            self._metadata.pop(handle.value, None)
        else:
            self._metadata[handle.value] = dict(metadata)

    # ------------------------------------------------------------------------- IVF
    @property
    def is_ivf(self) -> bool:
        return self.configuration.is_ivf

    @property
    def is_trained(self) -> bool:
        """Always true for a flat index (:349-352)."""
        return not self.is_ivf or self._centroids is not None

    def set_auto_training(self, enabled: bool) -> None:
        self._auto_train = bool(enabled)

    def train(self) -> None:
        """k-means over the live vectors (:396-446); a flat or trained index is left as is."""
        from .ivf import KMeansConfiguration, KMeansPipeline
        if not self.is_ivf or self._centroids is not None:
            return
        live = self._rows[~self._deleted]
        if live.shape[0] == 0:
            raise VAIndexError("Cannot train IVF index with no vectors")
        nlist = self.configuration.index_type[1]
        if live.shape[0] < nlist:
            raise VAIndexError(f"IVF training needs at least nlist ({nlist}) vectors, got {live.shape[0]}")
        cfg = KMeansConfiguration(num_clusters=nlist, dimension=self.configuration.dimension, max_iterations=25,
                                  convergence_threshold=1e-3)
        self._centroids = KMeansPipeline(self.context, cfg).fit(live).centroids
        self._ivf_dirty = True

    def _ivf_route(self, k: int) -> bool:
        cfg = self.configuration
        if not cfg.is_ivf or self._centroids is None or k > 128:
            return False
        return not (cfg.routing_threshold > 0 and self.count < cfg.routing_threshold)

    def _ivf_structure(self):
        import ctypes

        from .ivf import IVFGPUIndexStructure
        if self._ivf is None or self._ivf_dirty:
            if self._ivf is not None:
                self._ivf.close()
                self._ivf = None
            db = self._database()
            dc = self.context.get_buffer_for(self._centroids)
            h = ctypes.c_void_p()
            nlist = self._centroids.shape[0]
            _ffi.call("va_ivf_create", self.context.handle, db.rows_ptr(), self._rows.shape[0],
                      self.configuration.dimension, dc.ptr, nlist, 0, ctypes.byref(h))
            self._ivf = IVFGPUIndexStructure(self.context, h.value, nlist, self.configuration.dimension)
            self._ivf_dirty = False
        return self._ivf

    def _ivf_fetch(self, q: np.ndarray, fetch_k: int):
        from .ivf import IVFSearchConfiguration, IVFSearchPipeline
        st = self._ivf_structure()
        nlist, nprobe = self.configuration.index_type[1], self.configuration.index_type[2]
        res = IVFSearchPipeline(self.context, IVFSearchConfiguration(nlist, nprobe, self.configuration.dimension)) \
            .search(q, st, fetch_k)
        return res.distances, res.indices

    # ------------------------------------------------------------------------- queries on handles
    @property
    def count(self) -> int:
        return len(self._handle_slot)

    @property
    def allocated_slots(self) -> int:
        return self._rows.shape[0]

    def contains(self, handle: VectorHandle) -> bool:
        return handle.value in self._handle_slot

    def metadata(self, handle: VectorHandle) -> Optional[VectorMetadata]:
        return self._metadata.get(handle.value)

    def vector(self, handle: VectorHandle) -> Optional[np.ndarray]:
        slot = self._handle_slot.get(handle.value)
        return None if slot is None else self._rows[slot].copy()

    def all_handles(self) -> list[VectorHandle]:
        return [VectorHandle(h) for h, s in sorted(self._handle_slot.items(), key=lambda t: t[1])]

    def handles_where(self, predicate: Callable[[Optional[VectorMetadata]], bool]) -> list[VectorHandle]:
        return [h for h in self.all_handles() if predicate(self._metadata.get(h.value))]

    def slot(self, handle: VectorHandle) -> Optional[int]:
        return self._handle_slot.get(handle.value)

    def handle(self, slot: int) -> Optional[VectorHandle]:
        if 0 <= slot < len(self._slot_handle) and not self._deleted[slot]:
            return VectorHandle(self._slot_handle[slot])
        return None

    # ------------------------------------------------------------------------- search
    def _database(self) -> Database:
        if self._db is None:
            self._db = Database(self.context, self._rows)
        return self._db

    def _fetch(self, q: np.ndarray, fetch_k: int):
        """(values, slots) of the fetch_k (<= 4096) best slots per query row, best first, (value,
        slot) order: the fused search up to its k limit (1024), beyond it the device distance
        matrix and the device top-k selection."""
        from .kernels import MAXIMUM, MINIMUM, TopKSelectionKernel, _matrix
        metric = _METRICS[self.configuration.metric]
        if fetch_k <= _ffi.MAX_K:
            return knn_search_host(self.context, self._database(), q, fetch_k, metric, self.precision)
        m = _matrix(self.context, q, self._rows, metric, metric == _ffi.METRIC_COSINE)
        larger = metric == _ffi.METRIC_IP
        return TopKSelectionKernel(self.context).select_arrays(m, fetch_k, MAXIMUM if larger else MINIMUM)

    def _search_survivors(self, q: np.ndarray, k: int, filter: Filter, seen: set) -> list:  # noqa: A002
        """The filtered search's last step once the doubling fetch passes 4096 candidates (a very
        selective filter): the filter runs over every live slot not examined yet, and the exact
        device search runs over the rows that pass (a temporary database of those rows; ids map
        back to slots)."""
        live = np.nonzero(~self._deleted)[0]
        keep = []
        for s in live:
            if int(s) in seen:
                continue
            h = VectorHandle(self._slot_handle[int(s)])
            if filter(h, self._metadata.get(h.value)):
                keep.append(int(s))
        if not keep:
            return []
        slots = np.asarray(keep, np.int64)
        sub = Database(self.context, self._rows[slots])
        try:
            metric = _METRICS[self.configuration.metric]
            vals, ids = knn_search_host(self.context, sub, q, min(k, len(keep), _ffi.MAX_K), metric, self.precision)
        finally:
            sub.close()
        out = []
        for i, v in zip(ids[0], vals[0]):
            if int(i) != _ffi.INVALID_ID:
                s = int(slots[int(i)])
                out.append(IndexSearchResult(VectorHandle(self._slot_handle[s]), float(v)))
        return out

    def search(self, query, k: int, filter: Optional[Filter] = None) -> SearchResults:  # noqa: A002
        q = np.ascontiguousarray(query, np.float32)
        if q.ndim != 1:
            raise VAIndexError("search(query:) takes one vector; use search_batch")
        return self.search_batch(q[None, :], k, filter)[0]

    def search_batch(self, queries, k: int, filter: Optional[Filter] = None) -> list[SearchResults]:  # noqa: A002
        q = np.ascontiguousarray(queries, np.float32)
        if q.ndim != 2 or q.shape[1] != self.configuration.dimension:
            raise VAIndexError(f"dimension mismatch: expected {self.configuration.dimension}")
        if k <= 0:
            raise VAIndexError(f"k must be positive, got {k}")
        allocated = self._rows.shape[0]
        if allocated == 0 or self.count == 0:
            return [SearchResults([]) for _ in range(q.shape[0])]
        deleted = int(self._deleted.sum())
        ivf = self._ivf_route(k)
        if filter is not None:
            if ivf and q.shape[0] == 1:
                return [self._search_ivf_filtered(q, k, filter)]
            return [self._search_filtered(q[r:r + 1], k, filter) for r in range(q.shape[0])]
        if ivf:
            vals, ids = self._ivf_fetch(q, min(k + deleted, 128))
        else:
            vals, ids = self._fetch(q, min(k + deleted, allocated))
        out = []
        for r in range(q.shape[0]):
            res = []
            for i, v in zip(ids[r], vals[r]):
                i = int(i)
                if i == _ffi.INVALID_ID or self._deleted[i]:
                    continue
                res.append(IndexSearchResult(VectorHandle(self._slot_handle[i]), float(v)))
                if len(res) == k:
                    break
            out.append(SearchResults(res, candidates_searched=allocated, is_exhaustive=not ivf))
        return out

    def _search_ivf_filtered(self, q: np.ndarray, k: int, filter: Filter) -> SearchResults:  # noqa: A002
        """searchIVF with a filter (:1397-1420): over-fetch 3k (at most 128), skip deleted slots,
        keep what passes the filter."""
        vals, ids = self._ivf_fetch(q, min(3 * k, 128))
        res = []
        for i, v in zip(ids[0], vals[0]):
            i = int(i)
            if i == _ffi.INVALID_ID or self._deleted[i]:
                continue
            h = VectorHandle(self._slot_handle[i])
            if filter(h, self._metadata.get(h.value)):
                res.append(IndexSearchResult(h, float(v)))
                if len(res) >= k:
                    break
        return SearchResults(res, candidates_searched=self.count, is_exhaustive=False)

    def _search_filtered(self, q: np.ndarray, k: int, filter: Filter) -> SearchResults:  # noqa: A002
        """searchFiltered (:1188-1265): fetch 2k, double until k results pass the filter or every
        slot has been examined; slots already seen are skipped."""
        allocated = self._rows.shape[0]
        fetch_k = min(2 * k, allocated)
        results: list[IndexSearchResult] = []
        seen: set[int] = set()
        while len(results) < k:
            vals, ids = self._fetch(q, fetch_k)
            for i, v in zip(ids[0], vals[0]):
                i = int(i)
                if i == _ffi.INVALID_ID or i in seen:
                    continue
                seen.add(i)
                if self._deleted[i]:
                    continue
                h = VectorHandle(self._slot_handle[i])
                if filter(h, self._metadata.get(h.value)):
                    results.append(IndexSearchResult(h, float(v)))
                    if len(results) >= k:
                        break
            if len(results) >= k:
                break
            nxt = min(fetch_k * 2, allocated)
            if nxt == fetch_k or len(seen) >= allocated:
                break
            if nxt > _ffi.MAX_SELECT_K:
                # every later candidate passes the filter first; the device search orders them
                results.extend(self._search_survivors(q, k - len(results), filter, seen))
                return SearchResults(results[:k], candidates_searched=allocated, is_exhaustive=True)
            fetch_k = nxt
        return SearchResults(results, candidates_searched=len(seen), is_exhaustive=True)
