"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is a C++ restatement of VectorAccelerate's CPU search arithmetic (see
``va_oracle.cpp`` for the reference file:line each function follows). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this module, and
only as the checker or the timed CPU baseline: the product library never calls it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

METRIC_L2, METRIC_COSINE, METRIC_IP = 0, 1, 2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_U64 = ctypes.c_uint64
_U32 = ctypes.c_uint32


def build() -> None:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "orc_gen_gaussian": [_P, _I64, _I, _U64, _I64, _I],
            "orc_gen_mixture": [_P, _I64, _I, _U64, _I64, _I, _F, _I, _I],
            "orc_knn": [_P, _I64, _P, _I, _I64, _I, _I, _I, _I, _I, _P, _P],
            "orc_rerank": [_P, _I64, _P, _I, _I, _P, _I, _I, _I, _I, _P, _P],
            "orc_topk_select": [_P, _I64, _I64, _I64, _I, _I, _I, _P, _P],
            "orc_topk_merge": [_P, _P, _I, _P, _P, _I, _U32, _I64, _I, _P, _P],
            "orc_l2_pairs": [_P, _P, _I64, _I, _I, _P],
            "orc_cosine_pairs": [_P, _P, _I64, _I, _I, _P],
            "orc_matrix": [_P, _I64, _P, _I64, _I, _I, _I, _I, _P, _I64],
            "orc_sq_params": [_P, _I64, _I, _I, _P],
            "orc_quantize_int8": [_P, _I64, _F, ctypes.c_int8, _P, _P, _I64, _I64, _P],
            "orc_dequantize_int8": [_P, _I64, _F, ctypes.c_int8, _P, _P, _I64, _I64, _P],
            "orc_quantize_int4": [_P, _I64, _F, ctypes.c_int8, _P],
            "orc_dequantize_int4": [_P, _I64, _F, ctypes.c_int8, _P],
            "orc_sq_perdim_params": [_P, _I64, _I, _P, _P],
            "orc_sq_perdim_quantize": [_P, _I64, _I, _P, _P, _P],
            "orc_int8_knn": [_P, _P, _I64, _P, _P, _I64, _I, _I, _I, _I, _P, _P, _P, _P],
            "orc_binary_quantize": [_P, _I64, _I, _F, _P],
            "orc_hamming_matrix": [_P, _I64, _P, _I64, _I, _P],
            "orc_hamming_knn": [_P, _I64, _P, _I64, _I, _I, _I, _P, _P],
            "orc_f32_to_bf16": [_P, _I64, _P],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        L.orc_sq_params.restype = _F
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------------------- data
def gen_gaussian(rows: int, dim: int, seed: int, row0: int = 0, threads: int = 0) -> np.ndarray:
    out = np.empty((rows, dim), np.float32)
    lib().orc_gen_gaussian(_ptr(out), rows, dim, seed, row0, threads)
    return out


def gen_mixture(rows: int, dim: int, seed: int, n_centroids: int, sigma: float, normalize: bool,
                row0: int = 0, threads: int = 0) -> np.ndarray:
    out = np.empty((rows, dim), np.float32)
    lib().orc_gen_mixture(_ptr(out), rows, dim, seed, row0, n_centroids, sigma, int(normalize), threads)
    return out


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_ptr(x), x.size, _ptr(out))
    return out


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- search
def knn(queries, database, k: int, metric: int = METRIC_L2, truth: bool = True, threads: int = 0,
        db_bf16: bool = False):
    """Exact k-NN. ``database`` is fp32 rows, or uint16 bf16 bit patterns when ``db_bf16``."""
    q = _c(queries, np.float32)
    x = _c(database, np.uint16 if db_bf16 else np.float32)
    Q, d = q.shape
    N = x.shape[0]
    ids = np.empty((Q, k), np.uint32)
    vals = np.empty((Q, k), np.float32)
    lib().orc_knn(_ptr(q), Q, _ptr(x), 1 if db_bf16 else 0, N, d, k, metric, 1 if truth else 0, threads,
                  _ptr(ids), _ptr(vals))
    return ids, vals


def rerank(queries, database, cand_ids, k: int, metric: int = METRIC_L2, threads: int = 0, db_bf16=False):
    q = _c(queries, np.float32)
    x = _c(database, np.uint16 if db_bf16 else np.float32)
    c = _c(cand_ids, np.uint32)
    Q, d = q.shape
    ids = np.empty((Q, k), np.uint32)
    vals = np.empty((Q, k), np.float32)
    lib().orc_rerank(_ptr(q), Q, _ptr(x), 1 if db_bf16 else 0, d, _ptr(c), c.shape[1], k, metric, threads,
                     _ptr(ids), _ptr(vals))
    return ids, vals


def topk_select(values, k: int, mode: int = 0, threads: int = 0):
    v = _c(values, np.float32)
    B, n = v.shape
    vals = np.empty((B, k), np.float32)
    ids = np.empty((B, k), np.uint32)
    lib().orc_topk_select(_ptr(v), B, n, n, k, mode, threads, _ptr(vals), _ptr(ids))
    return vals, ids


def topk_merge(run_vals, run_ids, chunk_vals, chunk_ids, chunk_base: int, mode: int = 0):
    rv, ri = _c(run_vals, np.float32), _c(run_ids, np.uint32)
    cv, ci = _c(chunk_vals, np.float32), _c(chunk_ids, np.uint32)
    Q, k = rv.shape
    kc = cv.shape[1]
    ov = np.empty((Q, k), np.float32)
    oi = np.empty((Q, k), np.uint32)
    lib().orc_topk_merge(_ptr(rv), _ptr(ri), k, _ptr(cv), _ptr(ci), kc, chunk_base, Q, mode, _ptr(ov), _ptr(oi))
    return ov, oi


def l2_pairs(a, b, compute_sqrt=False):
    a, b = _c(a, np.float32), _c(b, np.float32)
    out = np.empty(a.shape[0], np.float32)
    lib().orc_l2_pairs(_ptr(a), _ptr(b), a.shape[0], a.shape[1], int(compute_sqrt), _ptr(out))
    return out


def cosine_pairs(a, b, output_distance=False):
    a, b = _c(a, np.float32), _c(b, np.float32)
    out = np.empty(a.shape[0], np.float32)
    lib().orc_cosine_pairs(_ptr(a), _ptr(b), a.shape[0], a.shape[1], int(output_distance), _ptr(out))
    return out


def matrix(q, x, metric: int, flag: bool = False, threads: int = 0):
    q, x = _c(q, np.float32), _c(x, np.float32)
    out = np.empty((q.shape[0], x.shape[0]), np.float32)
    lib().orc_matrix(_ptr(q), q.shape[0], _ptr(x), x.shape[0], q.shape[1], metric, int(flag), threads,
                     _ptr(out), x.shape[0])
    return out


# ----------------------------------------------------------------------------- quantization
def sq_params(x, type_: int = 0, bits: int = 8):
    x = _c(x, np.float32).ravel()
    zp = ctypes.c_int8(0)
    s = lib().orc_sq_params(_ptr(x), x.size, type_, bits, ctypes.byref(zp))
    return float(s), int(zp.value)


def quantize_int8(x, scale, zero_point=0, scales=None, zps=None, n_channels=1):
    x = _c(x, np.float32).ravel()
    out = np.empty(x.size, np.int8)
    per = x.size // n_channels if scales is not None else 0
    sc = None if scales is None else _c(scales, np.float32)
    zp = None if zps is None else _c(zps, np.int8)
    lib().orc_quantize_int8(_ptr(x), x.size, scale, zero_point, _ptr(sc), _ptr(zp), per, n_channels, _ptr(out))
    return out


def dequantize_int8(c, scale, zero_point=0, scales=None, zps=None, n_channels=1):
    c = _c(c, np.int8).ravel()
    out = np.empty(c.size, np.float32)
    per = c.size // n_channels if scales is not None else 0
    sc = None if scales is None else _c(scales, np.float32)
    zp = None if zps is None else _c(zps, np.int8)
    lib().orc_dequantize_int8(_ptr(c), c.size, scale, zero_point, _ptr(sc), _ptr(zp), per, n_channels, _ptr(out))
    return out


def quantize_int4(x, scale, zero_point=0):
    x = _c(x, np.float32).ravel()
    out = np.empty((x.size + 1) // 2, np.uint8)
    lib().orc_quantize_int4(_ptr(x), x.size, scale, zero_point, _ptr(out))
    return out


def dequantize_int4(c, n, scale, zero_point=0):
    c = _c(c, np.uint8)
    out = np.empty(n, np.float32)
    lib().orc_dequantize_int4(_ptr(c), n, scale, zero_point, _ptr(out))
    return out


def sq_perdim_params(x):
    x = _c(x, np.float32)
    n, d = x.shape
    mins = np.empty(d, np.float32)
    scales = np.empty(d, np.float32)
    lib().orc_sq_perdim_params(_ptr(x), n, d, _ptr(mins), _ptr(scales))
    return mins, scales


def sq_perdim_quantize(x, mins, scales):
    x = _c(x, np.float32)
    n, d = x.shape
    out = np.empty((n, d), np.int8)
    lib().orc_sq_perdim_quantize(_ptr(x), n, d, _ptr(_c(mins, np.float32)), _ptr(_c(scales, np.float32)), _ptr(out))
    return out


def int8_knn(qcodes, qf, xcodes, xf, kc: int, k: int, threads: int = 0):
    qc, xc = _c(qcodes, np.int8), _c(xcodes, np.int8)
    qf, xf = _c(qf, np.float32), _c(xf, np.float32)
    Q, d = qc.shape
    N = xc.shape[0]
    cids = np.empty((Q, kc), np.uint32)
    cd = np.empty((Q, kc), np.int32)
    ids = np.empty((Q, k), np.uint32)
    vals = np.empty((Q, k), np.float32)
    lib().orc_int8_knn(_ptr(qc), _ptr(qf), Q, _ptr(xc), _ptr(xf), N, d, kc, k, threads, _ptr(cids), _ptr(cd),
                       _ptr(ids), _ptr(vals))
    return ids, vals, cids, cd


def binary_quantize(x, threshold: float = 0.0):
    x = _c(x, np.float32)
    n, d = x.shape
    out = np.empty((n, (d + 31) // 32), np.uint32)
    lib().orc_binary_quantize(_ptr(x), n, d, threshold, _ptr(out))
    return out


def hamming_matrix(q, x):
    q, x = _c(q, np.uint32), _c(x, np.uint32)
    out = np.empty((q.shape[0], x.shape[0]), np.uint32)
    lib().orc_hamming_matrix(_ptr(q), q.shape[0], _ptr(x), x.shape[0], q.shape[1], _ptr(out))
    return out


def hamming_knn(q, x, k: int, threads: int = 0):
    q, x = _c(q, np.uint32), _c(x, np.uint32)
    Q, w = q.shape
    ids = np.empty((Q, k), np.uint32)
    ds = np.empty((Q, k), np.uint32)
    lib().orc_hamming_knn(_ptr(q), Q, _ptr(x), x.shape[0], w, k, threads, _ptr(ids), _ptr(ds))
    return ids, ds
