"""numpy restatement of the reference's IVF search and k-means (TEST INFRASTRUCTURE ONLY).

Only ``tests/`` may import this module, as the checker of ``va_ivf_*``; the product never
calls it. Distances are exact squared L2 in fp64 of the fp32 inputs, rounded to fp32; ordering is
(fp32 distance, id), ties to the smaller id, as the flat oracle.

Parity pin: the reference's IVF tests (Tests/VectorAccelerateTests/IVFTests.swift,
IVFValidationTests.swift) check recall against brute force and structural properties rather than
fixed vectors; the pins here are the same two facts, checked in ``tests/test_ivf_oracle.py``:
with nprobe = nlist the search equals the flat oracle's exact k-NN, and Lloyd iterations from
given centroids reach the means of their own assignment.
"""

from __future__ import annotations

import numpy as np


def _sqdist(q: np.ndarray, x: np.ndarray) -> np.ndarray:
    """[len(q) x len(x)] squared L2 in fp64 (expanded per pair, no norm trick)."""
    q64 = q.astype(np.float64)
    x64 = x.astype(np.float64)
    out = np.empty((q64.shape[0], x64.shape[0]), np.float64)
    for i in range(q64.shape[0]):
        d = x64 - q64[i]
        out[i] = np.einsum("ij,ij->i", d, d)
    return out


def _best(dist32: np.ndarray, ids: np.ndarray, k: int):
    """The k smallest (distance, id) pairs of one row, sorted; padded with (+inf, 0xFFFFFFFF)."""
    order = np.lexsort((ids, dist32))[:k]
    v = np.full(k, np.inf, np.float32)
    i = np.full(k, 0xFFFFFFFF, np.uint32)
    v[: order.size] = dist32[order]
    i[: order.size] = ids[order]
    return v, i


def assign(rows: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """Nearest centroid of every row, ties to the lower list (KMeansAssignKernel,
    Index/Kernels/Clustering/KMeansAssignKernel.swift; ClusteringShaders.metal assign)."""
    d = _sqdist(rows, centroids).astype(np.float32)
    return np.argmin(d, axis=1).astype(np.uint32)  # argmin returns the first (lowest) index


def build_lists(rows: np.ndarray, centroids: np.ndarray, id_base: int = 0):
    """Rows in list order (stable within a list), their ids, the list offsets."""
    a = assign(rows, centroids)
    order = np.argsort(a, kind="stable")
    counts = np.bincount(a, minlength=centroids.shape[0])
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return rows[order], (order + id_base).astype(np.uint32), offsets


def search(queries, centroids, list_rows, list_ids, offsets, k: int, nprobe: int):
    """IVFSearchPipeline.search (Index/Kernels/IVF/IVFSearchPipeline.swift:197-570): the nprobe
    nearest centroids by (distance, list id), then the exact k best (distance, id) over the rows
    of those lists."""
    q = np.asarray(queries, np.float32)
    cd = _sqdist(q, centroids).astype(np.float32)
    lists = np.arange(centroids.shape[0], dtype=np.uint32)
    nq = q.shape[0]
    out_v = np.empty((nq, k), np.float32)
    out_i = np.empty((nq, k), np.uint32)
    for qi in range(nq):
        probes = np.lexsort((lists, cd[qi]))[:nprobe]
        sel = np.concatenate([np.arange(offsets[p], offsets[p + 1]) for p in probes]) if nprobe else np.zeros(0, int)
        sel = sel.astype(np.int64)
        if sel.size:
            d = _sqdist(q[qi : qi + 1], list_rows[sel])[0].astype(np.float32)
        else:
            d = np.zeros(0, np.float32)
        out_v[qi], out_i[qi] = _best(d, list_ids[sel], k)
    return out_v, out_i


def kmeans(x: np.ndarray, init: np.ndarray, max_iters: int, tol: float):
    """Lloyd iterations (KMeansPipeline.fit, Index/Kernels/Clustering/KMeansPipeline.swift:165-230):
    assign, replace each centroid by the fp64 mean of its rows (an empty list keeps its centroid),
    stop once the largest Euclidean centroid movement is below tol
    (KMeansConvergenceKernel.swift:78-110). Returns (centroids fp32, iterations)."""
    c = np.array(init, np.float32, copy=True)
    x64 = x.astype(np.float64)
    it = 0
    while it < max_iters:
        a = assign(x, c)
        sums = np.zeros((c.shape[0], x.shape[1]), np.float64)
        np.add.at(sums, a, x64)
        cnt = np.bincount(a, minlength=c.shape[0])
        new = c.copy()
        nz = cnt > 0
        new[nz] = (sums[nz] / cnt[nz, None]).astype(np.float32)
        move = np.sqrt(float(np.max(((new.astype(np.float64) - c.astype(np.float64)) ** 2).sum(axis=1))))
        c = new
        it += 1
        if move < tol:
            break
    return c, it
