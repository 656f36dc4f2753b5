"""Error types mirroring the reference's thrown Swift errors.

``VectorError.invalidInput`` / ``bufferAllocationFailed`` / ``computeFailed`` (VectorCore, used
throughout e.g. Kernels/Metal4/FusedL2TopKKernel.swift:445-468) and
``IndexError.invalidInput(message:)`` (FusedL2TopKKernel.swift:52-85) map onto the C ABI's
status codes: VA_ERR_INVALID_ARG -> InvalidInput, VA_ERR_OOM -> BufferAllocationFailed,
VA_ERR_CUDA -> ComputeFailed, VA_ERR_TIMEOUT -> Timeout, VA_ERR_UNSUPPORTED -> Unsupported,
VA_ERR_NCCL -> CollectiveFailed.
"""

from __future__ import annotations


class VectorError(Exception):
    """Base of every error raised by this package."""


class InvalidInput(VectorError):
    """VectorError.invalidInput."""


class BufferAllocationFailed(VectorError):
    """VectorError.bufferAllocationFailed."""


class ComputeFailed(VectorError):
    """VectorError.computeFailed (the command buffer / CUDA stream reported an error)."""


class Timeout(ComputeFailed):
    """A bounded wait (host or device side) expired."""


class Unsupported(VectorError):
    """A parameter combination this build does not support."""


class CollectiveFailed(VectorError):
    """A collective (NCCL) step of a sharded search failed."""


class IndexError(InvalidInput):  # noqa: A001 - mirrors the reference's IndexError type name
    """IndexError.invalidInput(message:): parameter validation of the index / fused kernel."""


_BY_STATUS = {-1: InvalidInput, -2: BufferAllocationFailed, -3: ComputeFailed, -4: CollectiveFailed,
              -5: Timeout, -6: Unsupported}


def raise_for_status(status: int, message: str) -> None:
    raise _BY_STATUS.get(status, ComputeFailed)(message)
