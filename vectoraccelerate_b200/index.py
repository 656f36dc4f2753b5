"""AcceleratedVectorIndex: the flat-index caller of the fused search.

Mirrors Index/AcceleratedVectorIndex.swift for the flat path: ``insert`` returns a stable
``VectorHandle``; ``remove`` marks a slot deleted (lazy deletion, Index/Internal/DeletionMask.swift);
``search(query:k:)`` (:895-934) and ``search(queries:k:)`` (:947-1000) run the batch GPU search with
``fetchK = min(k + deletedCount, allocatedSlots)`` (:1330), drop deleted slots and map slot ->
handle (:1349-1371). Distances are squared L2 (the reference's index is euclidean-only,
:305-315); cosine and inner product are accepted here as an extension.

Rows live in a resident device database that is rebuilt from the host mirror when inserts or
compaction changed it (the reference's GPUVectorStorage writes through unified memory).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _ffi
from .context import GPUContext
from .errors import IndexError as VAIndexError
from .kernels import Database, knn_search_host

_METRICS = {"euclidean": _ffi.METRIC_L2SQ, "cosine": _ffi.METRIC_COSINE, "dot": _ffi.METRIC_IP}


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
    results: list

    @property
    def count(self) -> int:
        return len(self.results)


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
        self._slot_handle: list[int] = []
        self._next_handle = 0
        self._db: Database | None = None
        self._dirty = True

    # ------------------------------------------------------------------------- mutation
    def insert(self, vector) -> VectorHandle:
        return self.insert_batch([vector])[0]

    def insert_batch(self, vectors) -> list[VectorHandle]:
        v = np.ascontiguousarray(vectors, np.float32)
        if v.ndim == 1:
            v = v[None, :]
        if v.shape[1] != self.configuration.dimension:
            raise VAIndexError(f"dimension mismatch: expected {self.configuration.dimension}, got {v.shape[1]}")
        self._rows = np.concatenate([self._rows, v])
        self._deleted = np.concatenate([self._deleted, np.zeros(v.shape[0], bool)])
        handles = []
        for _ in range(v.shape[0]):
            self._slot_handle.append(self._next_handle)
            handles.append(VectorHandle(self._next_handle))
            self._next_handle += 1
        self._dirty = True
        return handles

    def remove(self, handle: VectorHandle) -> None:
        try:
            slot = self._slot_handle.index(handle.value)
        except ValueError:
            raise VAIndexError(f"unknown handle {handle.value}") from None
        self._deleted[slot] = True

    @property
    def count(self) -> int:
        return int((~self._deleted).sum())

    # ------------------------------------------------------------------------- search
    def _database(self) -> Database:
        if self._dirty or self._db is None:
            if self._db is not None:
                self._db.close()
            self._db = Database(self.context, self._rows)
            self._dirty = False
        return self._db

    def search(self, query, k: int) -> SearchResults:
        q = np.asarray(query, np.float32)
        if q.ndim != 1:
            raise VAIndexError("search(query:) takes one vector; use search_batch")
        return self.search_batch(q[None, :], k)[0]

    def search_batch(self, queries, k: int) -> list[SearchResults]:
        q = np.ascontiguousarray(queries, np.float32)
        if q.ndim != 2 or q.shape[1] != self.configuration.dimension:
            raise VAIndexError(f"dimension mismatch: expected {self.configuration.dimension}")
        if k <= 0:
            raise VAIndexError(f"k must be positive, got {k}")
        allocated = self._rows.shape[0]
        if allocated == 0 or self.count == 0:
            return [SearchResults([]) for _ in range(q.shape[0])]
        deleted = int(self._deleted.sum())
        fetch_k = min(k + deleted, allocated)
        vals, ids = knn_search_host(self.context, self._database(), q, fetch_k, _METRICS[self.configuration.metric],
                                    self.precision)
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
            out.append(SearchResults(res))
        return out
