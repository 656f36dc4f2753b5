"""ctypes binding of libva_cuda (the C ABI declared in include/va_cuda.h).

The library is built in-tree (``vectoraccelerate_b200/libva_cuda.so``). There is no fallback:
if it is missing or a call fails, an exception is raised.
"""

from __future__ import annotations

import ctypes
import os

from .errors import raise_for_status

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libva_cuda.so")

# Constants mirrored from va_cuda.h.
VA_OK = 0
METRIC_L2SQ, METRIC_COSINE, METRIC_IP = 0, 1, 2
IVF_INIT_KMEANSPP, IVF_INIT_GIVEN, IVF_INIT_RANDOM = 0, 1, 2
PREC_AUTO, PREC_FP32, PREC_TF32, PREC_BF16 = 0, 1, 2, 3
DTYPE_F32, DTYPE_BF16 = 0, 1
SELECT_MIN, SELECT_MAX = 0, 1
MAX_DIM, MAX_K, MAX_SELECT_K = 4096, 1024, 4096
NCCL_ID_BYTES = 128
INVALID_ID = 0xFFFFFFFF

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_PP = ctypes.POINTER(ctypes.c_void_p)


class VaConfig(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("timeout_ms", ctypes.c_uint), ("stream", ctypes.c_void_p)]


# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "va_last_error": [],
    "va_abi_version": [],
    "va_device_count": [ctypes.POINTER(ctypes.c_int)],
    "va_context_create": [ctypes.POINTER(VaConfig), _PP],
    "va_context_destroy": [_P],
    "va_context_stream": [_P, _PP],
    "va_synchronize": [_P],
    "va_last_gpu_time_ms": [_P, ctypes.POINTER(ctypes.c_float)],
    "va_last_search_times": [_P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)],
    "va_profile_start": [_P, _I],
    "va_profile_stop": [_P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int)],
    "va_buffer_alloc": [_P, _SZ, _PP],
    "va_buffer_free": [_P, _P],
    "va_host_alloc": [_P, _SZ, _PP],
    "va_host_free": [_P, _P],
    "va_buffer_upload": [_P, _P, _P, _SZ],
    "va_buffer_download": [_P, _P, _P, _SZ],
    "va_buffer_copy": [_P, _P, _P, _SZ],
    "va_l2_distance_pairs": [_P, _P, _P, _I64, _I, _I, _P],
    "va_cosine_pairs": [_P, _P, _P, _I64, _I, _I, _P],
    "va_distance_matrix": [_P, _P, _I64, _P, _I64, _I, _I, _I, _P, _I64],
    "va_topk_select": [_P, _P, _I64, _I64, _I64, _I, _I, _P, _P, _I64],
    "va_topk_merge": [_P, _P, _P, _I, _P, _P, _I, _U32, _I64, _I, _P, _P],
    "va_merge_shards": [_P, _P, _P, _I, _I64, _I, _I, _P, _P],
    "va_db_create": [_P, _P, _I, _I64, _I, _I, _U32, _PP],
    "va_db_append": [_P, _P, _P, _I, _I64],
    "va_db_update": [_P, _P, _I64, _P, _I, _I64],
    "va_db_compact": [_P, _P, _P, _P],
    "va_db_destroy": [_P],
    "va_db_info": [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I), ctypes.POINTER(_I)],
    "va_db_rows": [_P, _PP],
    "va_knn_search": [_P, _P, _P, _I64, _I, _I, _I, _I, _P, _P],
    "va_knn_search_host": [_P, _P, _P, _I64, _I, _I, _I, _I, _P, _P],
    "va_knn_search_noalloc": [_P, _P, _P, _I64, _I, _I, _I, _I, _P, _P],
    "va_last_search_stats": [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64)],
    "va_nccl_unique_id": [_P],
    "va_context_create_multi": [_P, _I, ctypes.POINTER(VaConfig), _PP],
    "va_context_create_rank": [ctypes.POINTER(VaConfig), _I, _I, _P, _PP],
    "va_context_group": [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)],
    "va_shard_range": [_P, _I64, _I, ctypes.POINTER(_I64), ctypes.POINTER(_I64)],
    "va_db_create_sharded": [_P, _P, _I, _I64, _I, _I, _PP],
    "va_db_create_int8_sharded": [_P, _P, _I, _I64, _I, _PP],
    "va_db_create_binary_sharded": [_P, _P, _I, _I64, _I, _PP],
    "va_db_shard": [_P, _I, _PP],
    "va_sq_quantize_int8": [_P, _P, _I64, _F, ctypes.c_int8, _P, _P, _I64, _P],
    "va_sq_dequantize_int8": [_P, _P, _I64, _F, ctypes.c_int8, _P, _P, _I64, _P],
    "va_sq_quantize_int4": [_P, _P, _I64, _F, ctypes.c_int8, _P],
    "va_sq_dequantize_int4": [_P, _P, _I64, _F, ctypes.c_int8, _P],
    "va_minmax": [_P, _P, _I64, _P],
    "va_sq_perdim_minmax": [_P, _P, _I64, _I, _P, _P],
    "va_db_create_int8": [_P, _P, _I, _I64, _I, _P, _P, _U32, _PP],
    "va_db_int8_params": [_P, _P, _P, _P, _P],
    "va_int8_knn_search": [_P, _P, _P, _I64, _I, _I, _P, _P],
    "va_binary_quantize": [_P, _P, _I64, _I, _F, _P],
    "va_hamming_matrix": [_P, _P, _I64, _P, _I64, _I, _P, _P, _I],
    "va_hamming_knn": [_P, _P, _I64, _P, _I64, _I, _I, _P, _P],
    "va_db_create_binary": [_P, _P, _I, _I64, _I, _U32, _PP],
    "va_db_binary_set_chunk_rows": [_P, _I64],
    "va_hamming_knn_db": [_P, _P, _P, _I64, _I, _P, _P],
    "va_ivf_train": [_P, _P, _I64, _I, _I, _I, _F, _U64, _I, _P, _P],
    "va_ivf_create": [_P, _P, _I64, _I, _P, _I, _U32, _PP],
    "va_ivf_create_lists": [_P, _P, _I, _I, _P, _P, _P, _I, _PP],
    "va_ivf_destroy": [_P],
    "va_ivf_list_sizes": [_P, _P],
    "va_ivf_search": [_P, _P, _P, _I64, _I, _I, _P, _P],
    "va_ivf_search_host": [_P, _P, _P, _I64, _I, _I, _P, _P],
    "va_gen_gaussian": [_P, _P, _I64, _I, _U64, _I64],
    "va_gen_mixture": [_P, _P, _I64, _I, _U64, _I64, _I, _F, _I],
    "va_f32_to_bf16": [_P, _P, _I64, _P],
}
_RESTYPES = {"va_last_error": ctypes.c_char_p, "va_abi_version": ctypes.c_int}

_lib = None


def load() -> ctypes.CDLL:
    """Load libva_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m vectoraccelerate_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().va_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Call an ABI function and raise the mapped exception on a non-zero status."""
    status = getattr(load(), name)(*args)
    if status != VA_OK:
        raise_for_status(status, f"{name}: {last_error()}")
