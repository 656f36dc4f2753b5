"""Row-sharded flat search across GPUs of one node.

The product path is the C ABI: ``GPUContext.rank`` (va_context_create_rank, one process per GPU)
or ``GPUContext.multi`` (va_context_create_multi, every device in one process) with a
``ShardedDatabase`` (va_db_create_sharded): every library search then searches each shard,
exchanges the per-shard top-k lists in one NCCL all-gather of packed (value, id) records and
merges them on the device. The reference is single-GPU; this is the build's multi-GPU layer.

This module keeps the shard arithmetic (``shard_bounds``, the same split as va_shard_range) and a
restatement of the exchange over torch.distributed (``ShardedSearch``: all-gather, then merge by
(distance, id)) whose ``local_search`` and ``merge`` are injectable, so the gather logic runs on
CPU with gloo in tests; ``merge_lists_host`` is its reference merge.
"""

from __future__ import annotations

from typing import Callable

import numpy as np


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first global row, row count) of ``rank``'s shard: N // world rows each, the last rank
    also takes the remainder."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    per = n // world
    row0 = rank * per
    return row0, (per if rank < world - 1 else n - row0)


class ShardedSearch:
    """Gather-and-merge driver. ``local_search(nq, k) -> (vals[nq,k], ids[nq,k])`` returns the
    shard's exact top-k with global ids; ``merge(gv[w,nq,k], gi[w,nq,k]) -> (vals, ids)``."""

    def __init__(self, world: int, local_search: Callable, merge: Callable, group=None):
        self.world = world
        self.local_search = local_search
        self.merge = merge
        self.group = group

    def search(self, nq: int, k: int):
        import torch
        import torch.distributed as dist
        lv, li = self.local_search(nq, k)
        if self.world == 1:
            return lv, li
        # Output concatenated along dim 0 (the form every backend accepts), viewed per rank.
        gv = torch.empty((self.world * lv.shape[0],) + tuple(lv.shape[1:]), dtype=lv.dtype, device=lv.device)
        gi = torch.empty((self.world * li.shape[0],) + tuple(li.shape[1:]), dtype=li.dtype, device=li.device)
        dist.all_gather_into_tensor(gv, lv.contiguous(), group=self.group)
        dist.all_gather_into_tensor(gi, li.contiguous(), group=self.group)
        return self.merge(gv.view((self.world,) + tuple(lv.shape)), gi.view((self.world,) + tuple(li.shape)))


def device_merge(context, world: int, nq: int, k: int, mode: int = 0):
    """Merge callable over libva_cuda's va_merge_shards (torch CUDA tensors in and out)."""
    import torch

    from . import _ffi

    def merge(gv, gi):
        fv = torch.empty((nq, k), dtype=torch.float32, device=gv.device)
        fi = torch.empty((nq, k), dtype=torch.int32, device=gv.device)
        _ffi.call("va_merge_shards", context.handle, gv.data_ptr(), gi.data_ptr(), world, nq, k, mode,
                  fv.data_ptr(), fi.data_ptr())
        return fv, fi

    return merge


def merge_lists_host(gv: np.ndarray, gi: np.ndarray, mode: int = 0):
    """Reference merge on the host (used only by CPU tests of the gather logic)."""
    w, nq, k = gv.shape
    vals = np.empty((nq, k), np.float32)
    ids = np.empty((nq, k), np.uint32)
    for q in range(nq):
        cand = [(float(gv[s, q, j]), int(gi[s, q, j])) for s in range(w) for j in range(k)
                if int(gi[s, q, j]) != 0xFFFFFFFF]
        cand.sort(key=(lambda t: (-t[0], t[1])) if mode else (lambda t: (t[0], t[1])))
        cand = cand[:k]
        pad = -np.inf if mode else np.inf
        cand += [(pad, 0xFFFFFFFF)] * (k - len(cand))
        vals[q] = [c[0] for c in cand]
        ids[q] = [c[1] for c in cand]
    return vals, ids
