"""GPUContext: the CUDA-backed replacement of the reference's Metal4Context.

Mirrors Core/Metal4Context.swift (``init(configuration:)`` :175-183, ``executeAndWait`` :342-410,
``getBuffer(size:)`` / ``getBuffer(for:)`` :471-488, ``lastGPUTiming`` :48-65) over the C ABI:
one CUDA device and one stream; buffers are device allocations owned by the caller
(``DeviceBuffer`` replaces MTLBuffer / BufferToken).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _ffi
from .errors import InvalidInput


@dataclass
class Metal4Configuration:
    """Context options (Metal4Configuration, Core/Metal4Context.swift:13-44)."""

    device: int = 0
    timeout_ms: int = 120_000
    stream: int | None = None  # optional external cudaStream_t (as an integer handle)


class DeviceBuffer:
    """A device allocation of ``nbytes`` with a dtype/shape view (MTLBuffer / BufferToken)."""

    def __init__(self, context: "GPUContext", nbytes: int, dtype=np.float32, shape=None):
        self.context = context
        self.nbytes = int(nbytes)
        self.dtype = np.dtype(dtype)
        self.shape = tuple(shape) if shape is not None else (self.nbytes // self.dtype.itemsize,)
        ptr = ctypes.c_void_p()
        _ffi.call("va_buffer_alloc", context.handle, ctypes.c_size_t(max(self.nbytes, 1)), ctypes.byref(ptr))
        self.ptr = ptr.value

    @property
    def address(self) -> int:
        return self.ptr

    def upload(self, array: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(array, dtype=self.dtype)
        if a.nbytes > self.nbytes:
            raise InvalidInput(f"upload of {a.nbytes} bytes into a {self.nbytes}-byte buffer")
        _ffi.call("va_buffer_upload", self.context.handle, self.ptr, a.ctypes.data_as(ctypes.c_void_p),
                  ctypes.c_size_t(a.nbytes))
        self.context.synchronize()
        return self

    def download(self, shape=None, dtype=None) -> np.ndarray:
        dt = np.dtype(dtype) if dtype is not None else self.dtype
        shp = tuple(shape) if shape is not None else self.shape
        out = np.empty(shp, dt)
        if out.nbytes > self.nbytes:
            raise InvalidInput(f"download of {out.nbytes} bytes from a {self.nbytes}-byte buffer")
        _ffi.call("va_buffer_download", self.context.handle, out.ctypes.data_as(ctypes.c_void_p), self.ptr,
                  ctypes.c_size_t(out.nbytes))
        self.context.synchronize()
        return out

    def free(self) -> None:
        if self.ptr:
            _ffi.call("va_buffer_free", self.context.handle, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            if self.ptr and self.context.handle:
                _ffi.load().va_buffer_free(self.context.handle, self.ptr)
        except Exception:
            pass


class GPUContext:
    """One CUDA device + stream. ``GPUContext()`` == ``Metal4Context()`` (aliased ``GPUContext``
    in the reference, VectorAccelerate.swift:254)."""

    def __init__(self, configuration: Metal4Configuration | None = None):
        cfg = configuration or Metal4Configuration()
        c = _ffi.VaConfig(cfg.device, cfg.timeout_ms, cfg.stream)
        h = ctypes.c_void_p()
        _ffi.call("va_context_create", ctypes.byref(c), ctypes.byref(h))
        self.handle = h.value
        self.configuration = cfg

    @classmethod
    def multi(cls, devices, timeout_ms: int = 120_000, stream: int | None = None) -> "GPUContext":
        """A group of devices in this process joined by an NCCL communicator
        (va_context_create_multi); the context lives on devices[0]."""
        devs = (ctypes.c_int * len(devices))(*devices)
        c = _ffi.VaConfig(devices[0], timeout_ms, stream)
        h = ctypes.c_void_p()
        _ffi.call("va_context_create_multi", devs, len(devices), ctypes.byref(c), ctypes.byref(h))
        self = cls.__new__(cls)
        self.handle = h.value
        self.configuration = Metal4Configuration(device=devices[0], timeout_ms=timeout_ms, stream=stream)
        return self

    @classmethod
    def rank(cls, nranks: int, rank: int, nccl_id: bytes, configuration: Metal4Configuration | None = None
             ) -> "GPUContext":
        """One rank of a group spread over processes (va_context_create_rank); every rank calls it
        with the same ``nccl_id`` (from ``nccl_unique_id()`` on one rank)."""
        cfg = configuration or Metal4Configuration()
        if len(nccl_id) != _ffi.NCCL_ID_BYTES:
            raise InvalidInput(f"nccl_id must be {_ffi.NCCL_ID_BYTES} bytes, got {len(nccl_id)}")
        c = _ffi.VaConfig(cfg.device, cfg.timeout_ms, cfg.stream)
        h = ctypes.c_void_p()
        idb = ctypes.create_string_buffer(bytes(nccl_id), _ffi.NCCL_ID_BYTES)
        _ffi.call("va_context_create_rank", ctypes.byref(c), nranks, rank, idb, ctypes.byref(h))
        self = cls.__new__(cls)
        self.handle = h.value
        self.configuration = cfg
        return self

    def group(self) -> tuple[int, int, int]:
        """(ranks in the group, global rank of this context's first device, local devices)."""
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _ffi.call("va_context_group", self.handle, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def shard_range(self, n: int, member: int = 0) -> tuple[int, int]:
        """(first row, rows) of an n-row database held by local device ``member``."""
        r0, cnt = ctypes.c_int64(), ctypes.c_int64()
        _ffi.call("va_shard_range", self.handle, n, member, ctypes.byref(r0), ctypes.byref(cnt))
        return r0.value, cnt.value

    @property
    def device(self) -> int:
        return self.configuration.device

    @property
    def stream(self) -> int:
        s = ctypes.c_void_p()
        _ffi.call("va_context_stream", self.handle, ctypes.byref(s))
        return s.value or 0

    def synchronize(self) -> None:
        """Bounded wait for the enqueued work (executeAndWait's completion + error check)."""
        _ffi.call("va_synchronize", self.handle)

    @property
    def last_gpu_time_ms(self) -> float:
        ms = ctypes.c_float()
        _ffi.call("va_last_gpu_time_ms", self.handle, ctypes.byref(ms))
        return float(ms.value)

    def last_search_stats(self) -> tuple[int, int]:
        """(queries the first tensor-core pass could not certify exact, queries that took the exact
        route) of the last fused search on this context."""
        u, e = ctypes.c_int64(), ctypes.c_int64()
        _ffi.call("va_last_search_stats", self.handle, ctypes.byref(u), ctypes.byref(e))
        return int(u.value), int(e.value)

    def get_buffer(self, size: int, dtype=np.float32, shape=None) -> DeviceBuffer:
        """getBuffer(size:) -- an uninitialised device buffer of ``size`` bytes."""
        return DeviceBuffer(self, size, dtype, shape)

    def get_buffer_for(self, array: np.ndarray, dtype=None) -> DeviceBuffer:
        """getBuffer(for:) -- a device buffer holding a copy of ``array``."""
        a = np.ascontiguousarray(array, dtype=dtype if dtype is not None else array.dtype)
        return DeviceBuffer(self, a.nbytes, a.dtype, a.shape).upload(a)

    def close(self) -> None:
        if getattr(self, "handle", None):
            _ffi.call("va_context_destroy", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                _ffi.load().va_context_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


Metal4Context = GPUContext


def nccl_unique_id() -> bytes:
    """An NCCL unique id (va_nccl_unique_id) for GPUContext.rank, shared by all ranks."""
    buf = ctypes.create_string_buffer(_ffi.NCCL_ID_BYTES)
    _ffi.call("va_nccl_unique_id", buf)
    return buf.raw
