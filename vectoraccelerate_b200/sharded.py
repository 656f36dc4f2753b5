"""Row-sharded flat search across GPUs of one node (one process per GPU).

The reference is single-GPU; this is the build's multi-GPU layer for the same search. Each rank
holds rows [row0, row0 + n_local) of the database (``shard_bounds``) with global ids
row0 + local row, searches them exactly, and the per-rank top-k lists are all-gathered
(torch.distributed: NCCL on GPUs, gloo on CPU) and merged with the (distance, id) order. Every
rank's list is already exact, so the merged list is exact.

``local_search`` and ``merge`` are injectable so the gather logic runs on CPU in tests; the
defaults call libva_cuda (``va_knn_search`` on the shard, ``va_merge_shards`` on the gathered
lists).
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
