"""MetalComputeProvider: the VectorCore-facing caller of the search kernels.

Mirrors Integration/MetalComputeProvider.swift (:112-259): ``batch_distance`` (distance from one
query to every candidate, in candidate order) and ``find_nearest`` (the k nearest as
(index, distance), nearest first), plus the batched ``find_nearest_batch``. Metric semantics
follow the reference: euclidean -> L2 distance (the square root of the squared distance),
cosine -> 1 - similarity (0 similarity for a zero norm), dotProduct -> raw dot product, where
larger is nearer. Every supported metric runs on the GPU: the reference sends dot products to
Accelerate on the CPU (:139-140) and this build has no CPU path, so manhattan and chebyshev (CPU
only in the reference, :142-148) raise ``Unsupported``. Equal distances keep the smaller index.
"""

from __future__ import annotations

import numpy as np

from . import _ffi
from .context import GPUContext
from .errors import InvalidInput, Unsupported
from .kernels import Database, _matrix, knn_search_host

SUPPORTED = ("euclidean", "cosine", "dotProduct")


class MetalComputeProvider:
    def __init__(self, context: GPUContext | None = None, precision: int = _ffi.PREC_AUTO):
        self.context = context or GPUContext()
        self.precision = precision

    @staticmethod
    def _check(query, candidates):
        q = np.ascontiguousarray(query, np.float32)
        x = np.ascontiguousarray(candidates, np.float32)
        if x.size == 0:
            return q, None
        if x.ndim != 2 or q.shape[-1] != x.shape[1]:
            raise InvalidInput(f"All candidates must match the query dimension ({q.shape[-1]})")
        return q, x

    @staticmethod
    def _metric(metric: str) -> int:
        if metric == "euclidean":
            return _ffi.METRIC_L2SQ
        if metric == "cosine":
            return _ffi.METRIC_COSINE
        if metric == "dotProduct":
            return _ffi.METRIC_IP
        if metric in ("manhattan", "chebyshev"):
            raise Unsupported(f"metric {metric!r} has no GPU kernel in this build (CPU-only in the reference)")
        raise InvalidInput(f"unknown metric {metric!r}")

    def batch_distance(self, query, candidates, metric: str) -> np.ndarray:
        """batchDistance(query:candidates:metric:) (:117-149): distances in candidate order."""
        q, x = self._check(query, candidates)
        if x is None:
            return np.zeros(0, np.float32)
        m = self._metric(metric)
        # flag: sqrt for euclidean, 1 - similarity for cosine, raw (not absolute) dot
        flag = metric in ("euclidean", "cosine")
        return _matrix(self.context, q.reshape(1, -1), x, m, flag)[0]

    def find_nearest_batch(self, queries, candidates, k: int, metric: str) -> list:
        """find_nearest for several queries against one candidate set, one fused GPU search."""
        q, x = self._check(queries, candidates)
        if k <= 0 or x is None:
            return [[] for _ in range(q.shape[0] if q.ndim == 2 else 1)]
        m = self._metric(metric)
        q2 = q.reshape(-1, x.shape[1])
        kk = min(k, x.shape[0])
        db = Database(self.context, x)
        try:
            vals, ids = knn_search_host(self.context, db, q2, kk, m, self.precision)
        finally:
            db.close()
        if metric == "euclidean":
            vals = np.sqrt(np.maximum(vals, 0.0))
        return [[(int(i), float(v)) for i, v in zip(ids[r], vals[r]) if int(i) != _ffi.INVALID_ID]
                for r in range(q2.shape[0])]

    def find_nearest(self, query, candidates, k: int, metric: str) -> list:
        """findNearest(query:in:k:metric:) (:162-194): up to k (index, distance), nearest first."""
        return self.find_nearest_batch(np.ascontiguousarray(query, np.float32).reshape(1, -1), candidates, k,
                                       metric)[0]
