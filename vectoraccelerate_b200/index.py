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
    """IndexConfiguration.flat(dimension:metric:capacity:) (Index/Types/IndexConfiguration.swift:330-345)."""

    dimension: int
    metric: str = "euclidean"
    capacity: int = 1024

    @staticmethod
    def flat(dimension: int, metric: str = "euclidean", capacity: int = 1024) -> "IndexConfiguration":
        return IndexConfiguration(dimension, metric, capacity)


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
        self._rows = np.zeros((0, configuration.dimension), np.float32)
        self._deleted = np.zeros(0, bool)
        self._slot_handle: list[int] = []          # slot -> handle value
        self._handle_slot: dict[int, int] = {}     # live handle value -> slot
        self._metadata: dict[int, VectorMetadata] = {}
        self._next_handle = 0
        self._db: Database | None = None

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
        slot0 = self._rows.shape[0]
        self._rows = np.concatenate([self._rows, v])
        self._deleted = np.concatenate([self._deleted, np.zeros(v.shape[0], bool)])
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
        return handles

    def remove(self, handle: VectorHandle) -> None:
        slot = self._handle_slot.pop(handle.value, None)
        if slot is None:
            raise VAIndexError(f"unknown handle {handle.value}")
        self._deleted[slot] = True
        self._metadata.pop(handle.value, None)

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
        self._rows = np.ascontiguousarray(self._rows[keep])
        self._slot_handle = [h for h, k in zip(self._slot_handle, keep) if k]
        self._handle_slot = {h: s for s, h in enumerate(self._slot_handle)}
        self._deleted = np.zeros(self._rows.shape[0], bool)

    def set_metadata(self, metadata: Optional[VectorMetadata], handle: VectorHandle) -> None:
        if handle.value not in self._handle_slot:
            raise VAIndexError(f"unknown handle {handle.value}")
        if metadata is None:
            self._metadata.pop(handle.value, None)
        else:
            self._metadata[handle.value] = dict(metadata)

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
        """(values, slots) of the fetch_k best slots per query row, best first, (value, slot)
        order: the fused search up to its k limit (1024), beyond it the device distance matrix
        and the device top-k selection (up to 4096); past that (a filtered search that has
        examined 4096 candidates without finding k) the device-computed distance row is ordered
        on the host."""
        from .kernels import MAXIMUM, MINIMUM, TopKSelectionKernel, _matrix
        metric = _METRICS[self.configuration.metric]
        if fetch_k <= _ffi.MAX_K:
            return knn_search_host(self.context, self._database(), q, fetch_k, metric, self.precision)
        m = _matrix(self.context, q, self._rows, metric, metric == _ffi.METRIC_COSINE)
        larger = metric == _ffi.METRIC_IP
        if fetch_k <= _ffi.MAX_SELECT_K:
            return TopKSelectionKernel(self.context).select_arrays(m, fetch_k, MAXIMUM if larger else MINIMUM)
        order = np.argsort(-m if larger else m, axis=1, kind="stable")[:, :fetch_k]
        return np.take_along_axis(m, order, 1).astype(np.float32), order.astype(np.uint32)

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
        if filter is not None:
            return [self._search_filtered(q[r:r + 1], k, filter) for r in range(q.shape[0])]
        deleted = int(self._deleted.sum())
        fetch_k = min(k + deleted, allocated)
        vals, ids = self._fetch(q, fetch_k)
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
            out.append(SearchResults(res, candidates_searched=allocated))
        return out

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
            fetch_k = nxt
        return SearchResults(results, candidates_searched=len(seen), is_exhaustive=True)
