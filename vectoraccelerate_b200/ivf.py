"""IVF search and k-means training with the reference's pipeline names, over libva_cuda.

Mirrors ``KMeansPipeline`` (Index/Kernels/Clustering/KMeansPipeline.swift:102-240, configured by
``KMeansConfiguration``, ClusteringKernels.swift:62-130) and ``IVFSearchPipeline``
(Index/Kernels/IVF/IVFSearchPipeline.swift:45-600, configured by ``IVFSearchConfiguration``,
IVFKernels.swift:28-60). Squared L2 only, as the reference's IVF path. The compute is
``va_ivf_train`` / ``va_ivf_create`` / ``va_ivf_create_lists`` / ``va_ivf_search``: k-means
assignment and the coarse quantizer run on the fused exact k-NN, the probed lists are scanned
with exact squared L2, results are ordered by (distance, id).

Differences from the reference, on purpose: the k-means++ draws come from a seeded generator
(deterministic; the reference uses the system generator), and ``init="random"`` offers distinct
random rows instead; ``IVFSearchPipeline.build`` forms the lists by nearest-centroid assignment on
the device (the reference's callers form them on the host).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _ffi
from .context import GPUContext
from .errors import InvalidInput

_vp = ctypes.c_void_p


def _f32_2d(a, what: str) -> np.ndarray:
    x = np.ascontiguousarray(a, dtype=np.float32)
    if x.ndim != 2 or x.shape[0] == 0:
        raise InvalidInput(f"{what} must be a non-empty 2-D array")
    return x


@dataclass(frozen=True)
class KMeansConfiguration:
    """ClusteringKernels.swift:62-130 (same defaults and validation)."""

    num_clusters: int
    dimension: int
    max_iterations: int = 100
    convergence_threshold: float = 1e-4
    seed: int = 42
    init: str = "kmeans++"   # or "random" (distinct rows); given centroids go to fit()

    def __post_init__(self):
        if self.init not in ("kmeans++", "random"):
            raise InvalidInput(f"init must be 'kmeans++' or 'random', got {self.init!r}")
        if self.num_clusters < 1:
            raise InvalidInput(f"numClusters must be at least 1, got {self.num_clusters}")
        if self.dimension < 1:
            raise InvalidInput(f"dimension must be at least 1, got {self.dimension}")
        if self.max_iterations < 1:
            raise InvalidInput(f"maxIterations must be at least 1, got {self.max_iterations}")
        if not self.convergence_threshold > 0:
            raise InvalidInput(f"convergenceThreshold must be positive, got {self.convergence_threshold}")


@dataclass
class KMeansResult:
    centroids: np.ndarray      # [num_clusters x dimension] fp32
    assignments: np.ndarray    # [n] uint32, nearest centroid of each vector
    iterations: int
    converged: bool


class KMeansPipeline:
    """k-means on the device: ``fit(vectors)`` -> KMeansResult (KMeansPipeline.swift:102-240)."""

    def __init__(self, context: GPUContext, configuration: KMeansConfiguration):
        self.context = context
        self.configuration = configuration

    def fit(self, vectors, initial_centroids=None) -> KMeansResult:
        cfg = self.configuration
        x = _f32_2d(vectors, "vectors")
        if x.shape[1] != cfg.dimension:
            raise InvalidInput(f"dimension mismatch: expected {cfg.dimension}, got {x.shape[1]}")
        if cfg.num_clusters > x.shape[0]:
            raise InvalidInput(f"numClusters {cfg.num_clusters} exceeds the {x.shape[0]} vectors")
        ctx = self.context
        dx = ctx.get_buffer_for(x)
        dc = ctx.get_buffer(4 * cfg.num_clusters * cfg.dimension, np.float32, (cfg.num_clusters, cfg.dimension))
        iters = ctypes.c_int(0)
        init = _ffi.IVF_INIT_KMEANSPP if cfg.init == "kmeans++" else _ffi.IVF_INIT_RANDOM
        if initial_centroids is not None:
            c0 = _f32_2d(initial_centroids, "initial_centroids")
            if c0.shape != (cfg.num_clusters, cfg.dimension):
                raise InvalidInput(f"initial centroids must be {cfg.num_clusters} x {cfg.dimension}")
            dc.upload(c0)
            init = _ffi.IVF_INIT_GIVEN
        _ffi.call("va_ivf_train", ctx.handle, dx.ptr, x.shape[0], cfg.dimension, cfg.num_clusters,
                  cfg.max_iterations, ctypes.c_float(cfg.convergence_threshold), cfg.seed, init, dc.ptr,
                  ctypes.byref(iters))
        centroids = dc.download()
        assign = _assign(ctx, centroids, dx.ptr, x.shape[0])
        return KMeansResult(centroids=centroids, assignments=assign, iterations=iters.value,
                            converged=iters.value < cfg.max_iterations)


def _assign(ctx: GPUContext, centroids: np.ndarray, dx_ptr: int, n: int) -> np.ndarray:
    from .kernels import Database  # local: kernels imports nothing from here

    db = Database(ctx, centroids)
    try:
        ov = ctx.get_buffer(4 * n, np.float32, (n, 1))
        oi = ctx.get_buffer(4 * n, np.uint32, (n, 1))
        _ffi.call("va_knn_search", ctx.handle, db.handle, dx_ptr, n, 1, _ffi.METRIC_L2SQ, _ffi.PREC_AUTO, 0,
                  ov.ptr, oi.ptr)
        return oi.download()[:, 0].copy()
    finally:
        db.close()


@dataclass(frozen=True)
class IVFSearchConfiguration:
    """IVFKernels.swift:28-60: numCentroids, nprobe, dimension (metric: squared L2)."""

    num_centroids: int
    nprobe: int
    dimension: int

    def __post_init__(self):
        if self.num_centroids < 1:
            raise InvalidInput("numCentroids must be positive")
        if not 1 <= self.nprobe <= self.num_centroids:
            raise InvalidInput(f"nprobe must be in 1...numCentroids ({self.num_centroids}), got {self.nprobe}")
        if self.dimension < 1:
            raise InvalidInput("dimension must be positive")


class IVFGPUIndexStructure:
    """Device-resident lists (IVFSearchPipeline.swift:575-600): centroids, rows in list order,
    vector ids, list offsets."""

    def __init__(self, context: GPUContext, handle: int, num_centroids: int, dimension: int):
        self.context = context
        self.handle = handle
        self.num_centroids = num_centroids
        self.dimension = dimension
        sizes = np.zeros(num_centroids, np.int64)
        _ffi.call("va_ivf_list_sizes", handle, sizes.ctypes.data_as(_vp))
        self.list_sizes = sizes
        self.total_vectors = int(sizes.sum())

    def list_count(self, list_index: int) -> int:
        return int(self.list_sizes[list_index])

    def close(self):
        if getattr(self, "handle", None):
            _ffi.call("va_ivf_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                _ffi.load().va_ivf_destroy(self.handle)
        except Exception:
            pass


@dataclass
class IVFSearchResult:
    indices: np.ndarray    # [Q x k] uint32, 0xFFFFFFFF where fewer than k vectors were probed
    distances: np.ndarray  # [Q x k] fp32 squared L2, +inf padding

    def results(self, query_index: int):
        ids, d = self.indices[query_index], self.distances[query_index]
        keep = ids != _ffi.INVALID_ID
        return list(zip(ids[keep].tolist(), d[keep].tolist()))


class IVFSearchPipeline:
    """prepare_index_structure / build / search (IVFSearchPipeline.swift:110-570)."""

    def __init__(self, context: GPUContext, configuration: IVFSearchConfiguration):
        self.context = context
        self.configuration = configuration

    def prepare_index_structure(self, centroids, lists, dimension: int | None = None) -> IVFGPUIndexStructure:
        """From host lists (one array of vectors per centroid); a vector's id is its position in
        the concatenated lists, as in the reference."""
        c = _f32_2d(centroids, "centroids")
        dim = dimension or c.shape[1]
        if c.shape[1] != dim:
            raise InvalidInput(f"centroid dimension {c.shape[1]} != {dim}")
        if len(lists) != c.shape[0]:
            raise InvalidInput(f"Number of centroids ({c.shape[0]}) must match number of lists ({len(lists)})")
        parts, offsets = [], [0]
        for lst in lists:
            a = np.asarray(lst, dtype=np.float32).reshape(-1, dim) if len(lst) else np.zeros((0, dim), np.float32)
            parts.append(a)
            offsets.append(offsets[-1] + a.shape[0])
        rows = np.ascontiguousarray(np.concatenate(parts, axis=0))
        off = np.asarray(offsets, np.int64)
        h = ctypes.c_void_p()
        rp = rows.ctypes.data_as(_vp) if rows.shape[0] else None
        _ffi.call("va_ivf_create_lists", self.context.handle, c.ctypes.data_as(_vp), c.shape[0], dim, rp,
                  off.ctypes.data_as(_vp), None, 0, ctypes.byref(h))
        return IVFGPUIndexStructure(self.context, h.value, c.shape[0], dim)

    def build(self, vectors, centroids, id_base: int = 0) -> IVFGPUIndexStructure:
        """Lists formed on the device: each vector goes to its nearest centroid; ids are the row
        index + id_base."""
        x = _f32_2d(vectors, "vectors")
        c = _f32_2d(centroids, "centroids")
        if x.shape[1] != c.shape[1]:
            raise InvalidInput(f"vector dimension {x.shape[1]} != centroid dimension {c.shape[1]}")
        ctx = self.context
        dx, dc = ctx.get_buffer_for(x), ctx.get_buffer_for(c)
        h = ctypes.c_void_p()
        _ffi.call("va_ivf_create", ctx.handle, dx.ptr, x.shape[0], x.shape[1], dc.ptr, c.shape[0], id_base,
                  ctypes.byref(h))
        return IVFGPUIndexStructure(ctx, h.value, c.shape[0], x.shape[1])

    def search(self, queries, structure: IVFGPUIndexStructure, k: int) -> IVFSearchResult:
        q = _f32_2d(queries, "Queries")
        if k <= 0:
            raise InvalidInput("k must be positive")
        if q.shape[1] != structure.dimension:
            raise InvalidInput(f"query dimension {q.shape[1]} != index dimension {structure.dimension}")
        nprobe = min(self.configuration.nprobe, structure.num_centroids)
        ov = np.empty((q.shape[0], k), np.float32)
        oi = np.empty((q.shape[0], k), np.uint32)
        _ffi.call("va_ivf_search_host", self.context.handle, structure.handle, q.ctypes.data_as(_vp), q.shape[0], k,
                  nprobe, ov.ctypes.data_as(_vp), oi.ctypes.data_as(_vp))
        return IVFSearchResult(indices=oi, distances=ov)

    def search_device(self, queries_ptr: int, nq: int, structure: IVFGPUIndexStructure, k: int, out_values_ptr: int,
                      out_indices_ptr: int) -> None:
        """Device-resident form: queries [nq x dimension] fp32 and outputs [nq x k] in device
        memory (stream-ordered on the context's stream)."""
        nprobe = min(self.configuration.nprobe, structure.num_centroids)
        _ffi.call("va_ivf_search", self.context.handle, structure.handle, queries_ptr, nq, k, nprobe, out_values_ptr,
                  out_indices_ptr)
