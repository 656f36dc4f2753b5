"""Kernel primitives with the reference's class names, over libva_cuda.

Each class mirrors one Swift kernel of Sources/VectorAccelerate/Kernels/Metal4/ (cited per class):
constructed from a context (``init(context:)``), with the high-level methods that take host
arrays (the reference's ``[[Float]]``) and device-buffer ``execute`` methods. Method names are the
Swift ones in snake_case. Results follow the reference's conventions: uint32 indices with
0xFFFFFFFF padding (skipped when converting to lists), squared L2 ascending, ``maximum`` mode
descending, ties by smaller index.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _ffi
from .context import DeviceBuffer, GPUContext
from .errors import IndexError as VAIndexError
from .errors import InvalidInput

_vp = ctypes.c_void_p


def _f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    if a.ndim == 1:
        a = a[None, :]
    return a


def _pairs_list(ids: np.ndarray, vals: np.ndarray, key: str = "distance"):
    out = []
    for r in range(ids.shape[0]):
        row = []
        for i, v in zip(ids[r], vals[r]):
            if int(i) != _ffi.INVALID_ID:
                row.append((int(i), float(v)))
        out.append(row)
    return out


class _Kernel:
    def __init__(self, context: GPUContext):
        self.context = context

    @property
    def _h(self):
        return self.context.handle


# ------------------------------------------------------------------------------------------ distance
class L2DistanceKernel(_Kernel):
    """L2DistanceKernel (L2DistanceKernel.swift:19-89): 1:1 pairs ``|a_i - b_i|`` (squared unless
    ``compute_sqrt``), plus the all-pairs matrix of l2_distance_kernel (L2Distance.metal:34-91)."""

    def encode(self, a: DeviceBuffer, b: DeviceBuffer, out: DeviceBuffer, pairs: int, dimension: int,
               compute_sqrt: bool = False) -> None:
        _ffi.call("va_l2_distance_pairs", self._h, a.ptr, b.ptr, pairs, dimension, int(compute_sqrt), out.ptr)

    def compute_pairs(self, a, b, compute_sqrt: bool = False) -> np.ndarray:
        a, b = _f32(a), _f32(b)
        if a.shape != b.shape:
            raise InvalidInput(f"pair shapes differ: {a.shape} vs {b.shape}")
        ctx = self.context
        da, db_ = ctx.get_buffer_for(a), ctx.get_buffer_for(b)
        out = ctx.get_buffer(4 * a.shape[0], np.float32, (a.shape[0],))
        self.encode(da, db_, out, a.shape[0], a.shape[1], compute_sqrt)
        return out.download()

    def distance_matrix(self, queries, dataset, compute_sqrt: bool = False) -> np.ndarray:
        return _matrix(self.context, queries, dataset, _ffi.METRIC_L2SQ, compute_sqrt)


class CosineSimilarityKernel(_Kernel):
    """CosineSimilarityKernel (CosineSimilarityKernel.swift:20-90): 1:1 pairs cosine similarity,
    or ``1 - sim`` when ``output_distance``; all-pairs matrix too."""

    def encode(self, a: DeviceBuffer, b: DeviceBuffer, out: DeviceBuffer, pairs: int, dimension: int,
               output_distance: bool = False) -> None:
        _ffi.call("va_cosine_pairs", self._h, a.ptr, b.ptr, pairs, dimension, int(output_distance), out.ptr)

    def compute_pairs(self, a, b, output_distance: bool = False) -> np.ndarray:
        a, b = _f32(a), _f32(b)
        if a.shape != b.shape:
            raise InvalidInput(f"pair shapes differ: {a.shape} vs {b.shape}")
        ctx = self.context
        da, db_ = ctx.get_buffer_for(a), ctx.get_buffer_for(b)
        out = ctx.get_buffer(4 * a.shape[0], np.float32, (a.shape[0],))
        self.encode(da, db_, out, a.shape[0], a.shape[1], output_distance)
        return out.download()

    def distance_matrix(self, queries, dataset, output_distance: bool = False) -> np.ndarray:
        return _matrix(self.context, queries, dataset, _ffi.METRIC_COSINE, output_distance)


class DotProductKernel(_Kernel):
    """DotProductKernel (DotProductKernel.swift:25-484): all-pairs dot products, optional
    absolute value; ``compute(queries:database:absoluteValue:)`` (:310-362)."""

    def compute(self, queries, database, absolute_value: bool = False) -> np.ndarray:
        return _matrix(self.context, queries, database, _ffi.METRIC_IP, absolute_value)


def _matrix(ctx: GPUContext, queries, dataset, metric: int, flag: bool) -> np.ndarray:
    q, x = _f32(queries), _f32(dataset)
    if q.shape[1] != x.shape[1]:
        raise InvalidInput("Dimension mismatch in input vectors")
    dq, dx = ctx.get_buffer_for(q), ctx.get_buffer_for(x)
    out = ctx.get_buffer(4 * q.shape[0] * x.shape[0], np.float32, (q.shape[0], x.shape[0]))
    _ffi.call("va_distance_matrix", ctx.handle, dq.ptr, q.shape[0], dx.ptr, x.shape[0], q.shape[1], metric,
              int(flag), out.ptr, x.shape[0])
    return out.download()


# ------------------------------------------------------------------------------------------ selection
MINIMUM, MAXIMUM = "minimum", "maximum"  # Metal4SelectionMode (TopKSelectionKernel.swift:23-29)


def _mode(mode) -> int:
    if mode in (MINIMUM, 0, _ffi.SELECT_MIN):
        return _ffi.SELECT_MIN
    if mode in (MAXIMUM, 1, _ffi.SELECT_MAX):
        return _ffi.SELECT_MAX
    raise InvalidInput(f"mode must be 'minimum' or 'maximum', got {mode!r}")


class TopKSelectionKernel(_Kernel):
    """TopKSelectionKernel (TopKSelectionKernel.swift:23-519) and WarpOptimizedSelectionKernel:
    batch top-k of value rows, minimum or maximum mode, sorted output."""

    maxK = _ffi.MAX_SELECT_K

    def execute(self, values: DeviceBuffer, batch: int, n: int, k: int, mode=MINIMUM, out_values=None,
                out_indices=None):
        ctx = self.context
        ov = out_values or ctx.get_buffer(4 * batch * k, np.float32, (batch, k))
        oi = out_indices or ctx.get_buffer(4 * batch * k, np.uint32, (batch, k))
        _ffi.call("va_topk_select", self._h, values.ptr, batch, n, n, k, _mode(mode), ov.ptr, oi.ptr, k)
        return ov, oi

    def select_arrays(self, values, k: int, mode=MINIMUM):
        """Top-k as (values [B,k], indices [B,k]) numpy arrays (padded rows keep the sentinel)."""
        v = _f32(values)
        if not (0 < k <= self.maxK):
            raise InvalidInput(f"K must be between 1 and {self.maxK}")
        dv = self.context.get_buffer_for(v)
        ov, oi = self.execute(dv, v.shape[0], v.shape[1], k, mode)
        return ov.download(), oi.download()

    def select(self, values, k: int, mode=MINIMUM, sorted: bool = True):  # noqa: A002
        """select(from:k:mode:sorted:) (:369-411) -> [[(index, value)]]; output is always sorted."""
        if len(values) == 0:
            return []
        vals, ids = self.select_arrays(values, k, mode)
        return _pairs_list(ids, vals)

    def select_single(self, values, k: int, mode=MINIMUM, sorted: bool = True):  # noqa: A002
        return self.select([values], k, mode, sorted)[0]


WarpOptimizedSelectionKernel = TopKSelectionKernel


class TopKMergeKernel(_Kernel):
    """TopKMergeKernel (TopKMergeKernel.swift:18-127): merge a running sorted top-k with a chunk's
    sorted top-kc whose indices are chunk-local (``chunk_base`` added)."""

    def merge(self, run_values, run_indices, chunk_values, chunk_indices, chunk_base: int, mode=MINIMUM):
        ctx = self.context
        rv, ri = _f32(run_values), np.ascontiguousarray(run_indices, np.uint32)
        cv, ci = _f32(chunk_values), np.ascontiguousarray(chunk_indices, np.uint32)
        q, k = rv.shape
        kc = cv.shape[1]
        drv, dri, dcv, dci = (ctx.get_buffer_for(a) for a in (rv, ri, cv, ci))
        ov = ctx.get_buffer(4 * q * k, np.float32, (q, k))
        oi = ctx.get_buffer(4 * q * k, np.uint32, (q, k))
        _ffi.call("va_topk_merge", self._h, drv.ptr, dri.ptr, k, dcv.ptr, dci.ptr, kc, chunk_base, q, _mode(mode),
                  ov.ptr, oi.ptr)
        return ov.download(), oi.download()


# ------------------------------------------------------------------------------------------ fused search
@dataclass(frozen=True)
class FusedL2TopKParameters:
    """FusedL2TopKParameters (FusedL2TopKKernel.swift:25-86) with this build's limits."""

    num_queries: int
    num_dataset: int
    dimension: int
    k: int

    maxK = _ffi.MAX_K
    maxDimension = _ffi.MAX_DIM

    def __post_init__(self):
        if self.num_queries <= 0:
            raise VAIndexError(f"numQueries must be positive, got {self.num_queries}")
        if self.num_dataset <= 0:
            raise VAIndexError(f"numDataset must be positive, got {self.num_dataset}")
        if self.dimension <= 0:
            raise VAIndexError(f"dimension must be positive, got {self.dimension}")
        if self.dimension > self.maxDimension:
            raise VAIndexError(f"dimension {self.dimension} exceeds maximum supported dimension {self.maxDimension}")
        if self.k <= 0:
            raise VAIndexError(f"k must be positive, got {self.k}")
        if self.k > self.maxK:
            raise VAIndexError(f"k {self.k} exceeds maximum supported k {self.maxK}")


@dataclass
class Metal4FusedL2Config:
    """Metal4FusedL2Config (FusedL2TopKKernel.swift:91-136), reduced to what applies here: the
    contraction precision and the rerank pool factor of the reduced-precision pass."""

    include_distances: bool = True
    precision: int = _ffi.PREC_AUTO
    rerank: int = 0


class Database:
    """A resident database (the storage buffer of GPUVectorStorage, Index/Internal/
    GPUVectorStorage.swift:52-100). Rows are fp32 or bf16 (uint16 bit patterns)."""

    def __init__(self, context: GPUContext, rows, dtype: int = _ffi.DTYPE_F32, id_base: int = 0,
                 device_ptr: int | None = None, n: int | None = None, dim: int | None = None):
        self.context = context
        h = ctypes.c_void_p()
        if device_ptr is not None:
            _ffi.call("va_db_create", context.handle, device_ptr, 1, n, dim, dtype, id_base, ctypes.byref(h))
            self.n, self.dim = n, dim
        else:
            a = np.ascontiguousarray(rows, dtype=np.uint16 if dtype == _ffi.DTYPE_BF16 else np.float32)
            if a.ndim != 2:
                raise InvalidInput("rows must be a 2-D array")
            _ffi.call("va_db_create", context.handle, a.ctypes.data_as(_vp), 0, a.shape[0], a.shape[1], dtype,
                      id_base, ctypes.byref(h))
            self.n, self.dim = a.shape
            context.synchronize()
        self.handle = h.value
        self.dtype = dtype
        self.id_base = id_base

    def rows_ptr(self) -> int:
        p = ctypes.c_void_p()
        _ffi.call("va_db_rows", self.handle, ctypes.byref(p))
        return p.value

    def _row_array(self, rows):
        a = np.ascontiguousarray(rows, dtype=np.uint16 if self.dtype == _ffi.DTYPE_BF16 else np.float32)
        if a.ndim == 1:
            a = a[None, :]
        if a.shape[1] != self.dim:
            raise InvalidInput(f"row dimension {a.shape[1]} != database dimension {self.dim}")
        return a

    def append(self, rows) -> None:
        """Append rows (va_db_append): capacity grows geometrically, derived data is updated."""
        a = self._row_array(rows)
        _ffi.call("va_db_append", self.context.handle, self.handle, a.ctypes.data_as(_vp), 0, a.shape[0])
        self.context.synchronize()
        self.n += a.shape[0]

    def update(self, slot0: int, rows) -> None:
        """Overwrite rows [slot0, slot0 + len(rows)) (va_db_update)."""
        a = self._row_array(rows)
        _ffi.call("va_db_update", self.context.handle, self.handle, slot0, a.ctypes.data_as(_vp), 0, a.shape[0])
        self.context.synchronize()

    def compact(self, keep) -> np.ndarray:
        """Keep rows where keep is true, in order (va_db_compact); returns old -> new slot (-1: dropped)."""
        k = np.ascontiguousarray(keep, np.uint8)
        if k.shape != (self.n,):
            raise InvalidInput(f"keep must have one entry per row ({self.n})")
        new_slot = np.empty(self.n, np.int64)
        _ffi.call("va_db_compact", self.context.handle, self.handle, k.ctypes.data_as(_vp), new_slot.ctypes.data_as(_vp))
        self.n = int((k != 0).sum())
        return new_slot

    def close(self):
        if getattr(self, "handle", None):
            _ffi.call("va_db_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                _ffi.load().va_db_destroy(self.handle)
        except Exception:
            pass


def knn_search_host(context: GPUContext, db: Database, queries: np.ndarray, k: int, metric: int = _ffi.METRIC_L2SQ,
                    precision: int = _ffi.PREC_AUTO, rerank: int = 0):
    """One whole search through the host-buffer entry point: returns (values, ids) numpy arrays."""
    q = _f32(queries)
    if q.shape[1] != db.dim:
        raise InvalidInput(f"query dimension {q.shape[1]} != database dimension {db.dim}")
    vals = np.empty((q.shape[0], k), np.float32)
    ids = np.empty((q.shape[0], k), np.uint32)
    _ffi.call("va_knn_search_host", context.handle, db.handle, q.ctypes.data_as(_vp), q.shape[0], k, metric,
              precision, rerank, vals.ctypes.data_as(_vp), ids.ctypes.data_as(_vp))
    return vals, ids


class FusedL2TopKKernel(_Kernel):
    """FusedL2TopKKernel (FusedL2TopKKernel.swift:205-1177): fused distance + top-k.

    ``execute`` takes device buffers (queries [Q x D] fp32 and a ``Database``) and returns device
    result buffers; ``find_nearest_neighbors`` is the high-level ``[[Float]]`` API (:439-529)."""

    def execute(self, queries: DeviceBuffer, dataset: Database, parameters: FusedL2TopKParameters,
                config: Metal4FusedL2Config | None = None, metric: int = _ffi.METRIC_L2SQ):
        cfg = config or Metal4FusedL2Config()
        ctx = self.context
        q, k = parameters.num_queries, parameters.k
        ov = ctx.get_buffer(4 * q * k, np.float32, (q, k))
        oi = ctx.get_buffer(4 * q * k, np.uint32, (q, k))
        _ffi.call("va_knn_search", self._h, dataset.handle, queries.ptr, q, k, metric, cfg.precision, cfg.rerank,
                  ov.ptr, oi.ptr)
        return Metal4FusedL2TopKResult(oi, ov if cfg.include_distances else None, q, k)

    def find_nearest_neighbors(self, queries, dataset, k: int, include_distances: bool = True,
                               config: Metal4FusedL2Config | None = None, metric: int = _ffi.METRIC_L2SQ):
        q, x = _f32(queries), _f32(dataset)
        if q.size == 0 or x.size == 0:
            raise InvalidInput("Empty input arrays")
        if q.shape[1] != x.shape[1]:
            raise InvalidInput("Dimension mismatch in input vectors")
        FusedL2TopKParameters(q.shape[0], x.shape[0], q.shape[1], k)
        cfg = config or Metal4FusedL2Config(include_distances=include_distances)
        db = Database(self.context, x)
        try:
            vals, ids = knn_search_host(self.context, db, q, k, metric, cfg.precision, cfg.rerank)
        finally:
            db.close()
        return _pairs_list(ids, vals)


@dataclass
class Metal4FusedL2TopKResult:
    """Metal4FusedL2TopKResult (FusedL2TopKKernel.swift:138-178)."""

    indices: DeviceBuffer
    distances: DeviceBuffer | None
    num_queries: int
    k: int

    def all_results(self):
        ids = self.indices.download()
        vals = self.distances.download() if self.distances is not None else np.zeros(ids.shape, np.float32)
        return _pairs_list(ids, vals)

    def results(self, query_index: int):
        if query_index >= self.num_queries:
            return []
        return self.all_results()[query_index]


# ------------------------------------------------------------------------------------------ quantization
@dataclass
class Metal4QuantizationResult:
    """Metal4QuantizationResult (ScalarQuantizationKernel.swift:103-140)."""

    quantized_data: bytes
    scale: float
    zero_point: int | None
    bit_width: int

    @property
    def compression_ratio(self) -> float:
        n = len(self.quantized_data) * (2 if self.bit_width == 4 else 1)
        return (4.0 * n) / max(1, len(self.quantized_data))


class ScalarQuantizationKernel(_Kernel):
    """ScalarQuantizationKernel (ScalarQuantizationKernel.swift:23-521): int8/int4, symmetric or
    asymmetric; parameters computed as computeQuantizationParams (:496-520) from a device min/max."""

    def _params(self, dx: DeviceBuffer, n: int, type_: str, bits: int):
        mm = self.context.get_buffer(8, np.float32, (2,))
        _ffi.call("va_minmax", self._h, dx.ptr, n, mm.ptr)
        mn, mx = (float(v) for v in mm.download())
        smax, amax = (7.0, 15.0) if bits == 4 else (127.0, 255.0)
        if type_ == "asymmetric":
            scale = float(np.float32(max(np.float32(mx - mn) / np.float32(amax), np.float32(1e-8))))
            # Int8(clamping: Int(-round(min / scale))) -- Swift round() is half away from zero.
            zp = int(min(127, max(-128, -_round_half_away(np.float32(mn) / np.float32(scale)))))
            return scale, zp
        absmax = max(abs(mn), abs(mx))
        scale = float(np.float32(max(np.float32(absmax) / np.float32(smax), np.float32(1e-8))))
        return scale, None

    def quantize(self, data, bit_width: int = 8, type: str = "symmetric") -> Metal4QuantizationResult:  # noqa: A002
        x = np.ascontiguousarray(data, np.float32).ravel()
        if x.size == 0:
            raise InvalidInput("Empty input")
        ctx = self.context
        dx = ctx.get_buffer_for(x)
        scale, zp = self._params(dx, x.size, type, bit_width)
        if bit_width == 8:
            out = ctx.get_buffer(x.size, np.int8, (x.size,))
            _ffi.call("va_sq_quantize_int8", self._h, dx.ptr, x.size, scale, zp or 0, None, None, 1, out.ptr)
        elif bit_width == 4:
            nb = (x.size + 1) // 2
            out = ctx.get_buffer(nb, np.uint8, (nb,))
            _ffi.call("va_sq_quantize_int4", self._h, dx.ptr, x.size, scale, zp or 0, out.ptr)
        else:
            raise InvalidInput(f"bit width must be 8 or 4, got {bit_width}")
        return Metal4QuantizationResult(out.download().tobytes(), scale, zp, bit_width)

    def dequantize(self, result: Metal4QuantizationResult, count: int) -> np.ndarray:
        ctx = self.context
        raw = np.frombuffer(result.quantized_data, np.uint8)
        din = ctx.get_buffer_for(raw)
        out = ctx.get_buffer(4 * count, np.float32, (count,))
        zp = result.zero_point or 0
        if result.bit_width == 8:
            _ffi.call("va_sq_dequantize_int8", self._h, din.ptr, count, result.scale, zp, None, None, 1, out.ptr)
        else:
            _ffi.call("va_sq_dequantize_int4", self._h, din.ptr, count, result.scale, zp, out.ptr)
        return out.download()


def _round_half_away(v) -> float:
    v = float(v)
    return float(np.floor(v + 0.5)) if v >= 0 else -float(np.floor(-v + 0.5))


# ------------------------------------------------------------------------------------------ binary
@dataclass
class Metal4BinaryVector:
    """Metal4BinaryVector (BinaryQuantizationKernel.swift:23-75): LSB-first packed words."""

    data: np.ndarray  # uint32 words
    dimension: int

    @property
    def num_words(self) -> int:
        return (self.dimension + 31) // 32

    def bit(self, index: int) -> bool:
        if not 0 <= index < self.dimension:
            return False
        return bool((int(self.data[index // 32]) >> (index % 32)) & 1)

    def hamming_distance(self, other: "Metal4BinaryVector") -> int:
        if self.dimension != other.dimension:
            return -1
        return int(sum(bin(int(a) ^ int(b)).count("1") for a, b in zip(self.data, other.data)))


class BinaryQuantizationKernel(_Kernel):
    """BinaryQuantizationKernel (BinaryQuantizationKernel.swift:23-513): sign binarisation
    (bit = value > threshold, threshold 0 as in the shader) and 1 x N Hamming distances."""

    def quantize_array(self, vectors, threshold: float = 0.0) -> np.ndarray:
        x = _f32(vectors)
        n, d = x.shape
        words = (d + 31) // 32
        dx = self.context.get_buffer_for(x)
        out = self.context.get_buffer(4 * n * words, np.uint32, (n, words))
        _ffi.call("va_binary_quantize", self._h, dx.ptr, n, d, threshold, out.ptr)
        return out.download()

    def quantize(self, vectors, threshold: float = 0.0):
        x = _f32(vectors)
        codes = self.quantize_array(x, threshold)
        return [Metal4BinaryVector(codes[i].copy(), x.shape[1]) for i in range(x.shape[0])]

    def compute_hamming_distances(self, query: Metal4BinaryVector, candidates) -> np.ndarray:
        """computeHammingDistances(query:candidates:) (:416-491): distances as float."""
        cand = np.stack([c.data for c in candidates]).astype(np.uint32)
        hk = HammingDistanceKernel(self.context)
        m = hk.compute_bit_packed(query.data[None, :].astype(np.uint32), cand, query.dimension)
        return m[0].astype(np.float32)


class HammingDistanceKernel(_Kernel):
    """HammingDistanceKernel (HammingDistanceKernel.swift:23-609): Q x N Hamming over packed
    words, bool-array helpers, and the fused k-NN (no materialised matrix)."""

    @staticmethod
    def pack_binary(bits) -> np.ndarray:
        """packBinary (:411-424): bit i -> word i/32, bit i%32."""
        b = np.asarray(bits, dtype=bool)
        words = (b.size + 31) // 32
        out = np.zeros(words, np.uint32)
        for i in np.nonzero(b)[0]:
            out[i // 32] |= np.uint32(1) << np.uint32(i % 32)
        return out

    def compute_bit_packed(self, queries: np.ndarray, dataset: np.ndarray, dimension: int | None = None,
                           normalized: bool = False) -> np.ndarray:
        q = np.ascontiguousarray(queries, np.uint32)
        x = np.ascontiguousarray(dataset, np.uint32)
        if q.ndim == 1:
            q = q[None, :]
        words = q.shape[1]
        ctx = self.context
        dq, dx = ctx.get_buffer_for(q), ctx.get_buffer_for(x)
        out = ctx.get_buffer(4 * q.shape[0] * x.shape[0], np.uint32, (q.shape[0], x.shape[0]))
        outn = ctx.get_buffer(4 * q.shape[0] * x.shape[0], np.float32, (q.shape[0], x.shape[0])) if normalized else None
        _ffi.call("va_hamming_matrix", self._h, dq.ptr, q.shape[0], dx.ptr, x.shape[0], words, out.ptr,
                  outn.ptr if outn else None, dimension or words * 32)
        return outn.download() if normalized else out.download()

    def distance_matrix(self, queries, dataset) -> np.ndarray:
        """distanceMatrix(queries:dataset:) over bool arrays -> float matrix."""
        q = np.stack([self.pack_binary(v) for v in queries])
        x = np.stack([self.pack_binary(v) for v in dataset])
        return self.compute_bit_packed(q, x).astype(np.float32)

    def nearest_neighbors(self, queries: np.ndarray, dataset: np.ndarray, k: int):
        """Fused Hamming k-NN -> (distances uint32 [Q,k], ids uint32 [Q,k])."""
        q = np.ascontiguousarray(queries, np.uint32)
        x = np.ascontiguousarray(dataset, np.uint32)
        ctx = self.context
        dq, dx = ctx.get_buffer_for(q), ctx.get_buffer_for(x)
        od = ctx.get_buffer(4 * q.shape[0] * k, np.uint32, (q.shape[0], k))
        oi = ctx.get_buffer(4 * q.shape[0] * k, np.uint32, (q.shape[0], k))
        _ffi.call("va_hamming_knn", self._h, dq.ptr, q.shape[0], dx.ptr, x.shape[0], q.shape[1], k, od.ptr, oi.ptr)
        return od.download(), oi.download()


class _DbHandle:
    def rows_ptr(self) -> int:
        """Device pointer of the stored rows: fp32 rows of an int8 database, packed codes of a binary one."""
        p = ctypes.c_void_p()
        _ffi.call("va_db_rows", self.handle, ctypes.byref(p))
        return p.value

    def close(self):
        if getattr(self, "handle", None):
            _ffi.call("va_db_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                _ffi.load().va_db_destroy(self.handle)
        except Exception:
            pass


class Int8Database(_DbHandle):
    """Resident int8 scalar-quantized database: per-dimension codes of fp32 rows plus the rows
    themselves for the exact rerank. Quantization: scale_j = max((max_j - min_j)/255, 1e-8),
    code = clamp(rint((x - min_j)/scale_j), 0, 255) - 128 (the asymmetric uint8 mapping of
    ScalarQuantizationKernel.swift:509-520 per dimension). `mins`/`maxs` fix the range (e.g. the
    global range of a sharded database); by default it is taken over these rows."""

    def __init__(self, context: GPUContext, rows=None, id_base: int = 0, mins=None, maxs=None,
                 device_ptr: int | None = None, n: int | None = None, dim: int | None = None):
        self.context = context
        h = ctypes.c_void_p()
        dmn = dmx = None
        if mins is not None:
            dmn = context.get_buffer_for(np.ascontiguousarray(mins, np.float32))
            dmx = context.get_buffer_for(np.ascontiguousarray(maxs, np.float32))
        pmn = dmn.ptr if dmn else None
        pmx = dmx.ptr if dmx else None
        if device_ptr is not None:
            _ffi.call("va_db_create_int8", context.handle, device_ptr, 1, n, dim, pmn, pmx, id_base, ctypes.byref(h))
            self.n, self.dim = n, dim
        else:
            a = _f32(rows)
            _ffi.call("va_db_create_int8", context.handle, a.ctypes.data_as(_vp), 0, a.shape[0], a.shape[1], pmn, pmx,
                      id_base, ctypes.byref(h))
            self.n, self.dim = a.shape
        context.synchronize()
        self.handle = h.value
        self.id_base = id_base

    def parameters(self):
        """(mins, scales) as numpy arrays."""
        pm, ps = ctypes.c_void_p(), ctypes.c_void_p()
        _ffi.call("va_db_int8_params", self.handle, ctypes.byref(pm), ctypes.byref(ps), None, None)
        mins = np.empty(self.dim, np.float32)
        scales = np.empty(self.dim, np.float32)
        _ffi.call("va_buffer_download", self.context.handle, mins.ctypes.data_as(_vp), pm.value,
                  ctypes.c_size_t(mins.nbytes))
        _ffi.call("va_buffer_download", self.context.handle, scales.ctypes.data_as(_vp), ps.value,
                  ctypes.c_size_t(scales.nbytes))
        self.context.synchronize()
        return mins, scales

    def codes(self) -> np.ndarray:
        """The int8 codes [n x dim]."""
        pc, stride = ctypes.c_void_p(), ctypes.c_int()
        _ffi.call("va_db_int8_params", self.handle, None, None, ctypes.byref(pc), ctypes.byref(stride))
        out = np.empty((self.n, stride.value), np.int8)
        _ffi.call("va_buffer_download", self.context.handle, out.ctypes.data_as(_vp), pc.value,
                  ctypes.c_size_t(out.nbytes))
        self.context.synchronize()
        return out[:, : self.dim].copy()

    def search(self, queries, k: int, candidates: int):
        """int8 L2 k-NN with exact rerank of `candidates` per query -> (values, ids) numpy."""
        q = _f32(queries)
        if q.shape[1] != self.dim:
            raise InvalidInput(f"query dimension {q.shape[1]} != database dimension {self.dim}")
        ctx = self.context
        dq = ctx.get_buffer_for(q)
        ov = ctx.get_buffer(4 * q.shape[0] * k, np.float32, (q.shape[0], k))
        oi = ctx.get_buffer(4 * q.shape[0] * k, np.uint32, (q.shape[0], k))
        _ffi.call("va_int8_knn_search", ctx.handle, self.handle, dq.ptr, q.shape[0], k, candidates, ov.ptr, oi.ptr)
        return ov.download(), oi.download()


class BinaryDatabase(_DbHandle):
    """Resident binary database of LSB-first packed codes (Metal4BinaryVector layout,
    BinaryQuantizationKernel.swift:23-74) searched by Hamming distance on the integer tensor
    cores; the same results as HammingDistanceKernel.nearest_neighbors."""

    def __init__(self, context: GPUContext, codes, dim_bits: int | None = None, id_base: int = 0):
        self.context = context
        c = np.ascontiguousarray(codes, np.uint32)
        if c.ndim != 2:
            raise InvalidInput("codes must be a 2-D array of uint32 words")
        self.n, self.words = c.shape
        self.dim_bits = dim_bits or self.words * 32
        h = ctypes.c_void_p()
        _ffi.call("va_db_create_binary", context.handle, c.ctypes.data_as(_vp), 0, self.n, self.dim_bits, id_base,
                  ctypes.byref(h))
        context.synchronize()
        self.handle = h.value
        self.id_base = id_base

    @classmethod
    def from_device(cls, context: GPUContext, codes_ptr: int, n: int, dim_bits: int, id_base: int = 0):
        """A database copied from packed codes already in device memory ([n x ceil(dim_bits/32)])."""
        self = cls.__new__(cls)
        self.context = context
        self.n, self.words, self.dim_bits = n, (dim_bits + 31) // 32, dim_bits
        h = ctypes.c_void_p()
        _ffi.call("va_db_create_binary", context.handle, codes_ptr, 1, n, dim_bits, id_base, ctypes.byref(h))
        context.synchronize()
        self.handle = h.value
        self.id_base = id_base
        return self

    def set_chunk_rows(self, rows: int):
        """Rows expanded per pass of batched searches (0: automatic); before the first search."""
        _ffi.call("va_db_binary_set_chunk_rows", self.handle, rows)

    def search(self, query_codes, k: int):
        """-> (distances uint32 [Q,k], ids uint32 [Q,k]), sorted by (distance, id)."""
        q = np.ascontiguousarray(query_codes, np.uint32)
        if q.ndim == 1:
            q = q[None, :]
        if q.shape[1] != self.words:
            raise InvalidInput(f"query words {q.shape[1]} != database words {self.words}")
        ctx = self.context
        dq = ctx.get_buffer_for(q)
        od = ctx.get_buffer(4 * q.shape[0] * k, np.uint32, (q.shape[0], k))
        oi = ctx.get_buffer(4 * q.shape[0] * k, np.uint32, (q.shape[0], k))
        _ffi.call("va_hamming_knn_db", ctx.handle, self.handle, dq.ptr, q.shape[0], k, od.ptr, oi.ptr)
        return od.download(), oi.download()


class ShardedDatabase(_DbHandle):
    """A row-sharded database over a group context (va_db_create_sharded, _int8_sharded,
    _binary_sharded): each rank holds rows [row0, row0 + rows) of the n-row database
    (``GPUContext.shard_range``). ``rows`` are the rows this process owns, in global order: all
    n rows for a multi-device context, this rank's shard for a rank context; a numpy array, or a
    device pointer with ``device_ptr``. Searched with the usual entry points (va_knn_search,
    va_int8_knn_search, va_hamming_knn_db), whose results are the whole database's."""

    def __init__(self, context: GPUContext, rows=None, n: int | None = None, dim: int | None = None,
                 kind: str = "float", dtype: int = _ffi.DTYPE_F32, device_ptr: int | None = None):
        self.context = context
        self.kind = kind
        if device_ptr is None:
            np_dt = np.uint32 if kind == "binary" else (np.uint16 if dtype == _ffi.DTYPE_BF16 else np.float32)
            a = np.ascontiguousarray(rows, dtype=np_dt)
            ptr, on_dev = a.ctypes.data_as(_vp), 0
            dim = dim or (a.shape[1] * 32 if kind == "binary" else a.shape[1])
            n = n or a.shape[0]
        else:
            ptr, on_dev = device_ptr, 1
        h = ctypes.c_void_p()
        if kind == "float":
            _ffi.call("va_db_create_sharded", context.handle, ptr, on_dev, n, dim, dtype, ctypes.byref(h))
        elif kind == "int8":
            _ffi.call("va_db_create_int8_sharded", context.handle, ptr, on_dev, n, dim, ctypes.byref(h))
        elif kind == "binary":
            _ffi.call("va_db_create_binary_sharded", context.handle, ptr, on_dev, n, dim, ctypes.byref(h))
        else:
            raise InvalidInput(f"kind must be float, int8 or binary, got {kind!r}")
        context.synchronize()
        self.handle = h.value
        self.n, self.dim, self.dtype = n, dim, dtype

    def rows_ptr(self, member: int = 0) -> int:
        """Device pointer of local device ``member``'s shard rows (codes for a binary database)."""
        sh = ctypes.c_void_p()
        _ffi.call("va_db_shard", self.handle, member, ctypes.byref(sh))
        p = ctypes.c_void_p()
        _ffi.call("va_db_rows", sh.value, ctypes.byref(p))
        return p.value
