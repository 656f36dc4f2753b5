"""The parity rule of the project (TEST INFRASTRUCTURE ONLY, like the rest of ``oracle/``).

Returned ids must equal the oracle's bit for bit, except where the two distances tie within 1e-5
relative; distances must agree within 1e-4 relative (fp32). Used by ``tests/`` (asserting),
``__graft_entry__.smoke()`` and ``bench.py``'s oracle-parity leg (counting).
"""

from __future__ import annotations

import numpy as np

REL_TIE = 1e-5
REL_DIST = 1e-4
INVALID = 0xFFFFFFFF


def true_values_at(gpu_ids, rerank_ids, rerank_vals):
    """The oracle's exact value of each GPU id at the GPU's position, from an oracle rerank of the
    GPU's ids (``oracle.rerank`` returns them sorted); NaN where an id is padding."""
    gpu_ids = np.asarray(gpu_ids).view(np.uint32)
    out = np.full(gpu_ids.shape, np.nan, np.float32)
    for r in range(gpu_ids.shape[0]):
        pos = {int(i): v for i, v in zip(rerank_ids[r], rerank_vals[r]) if int(i) != INVALID}
        for j, i in enumerate(gpu_ids[r]):
            if int(i) in pos:
                out[r, j] = pos[int(i)]
    return out


def summary(gpu_ids, gpu_vals, ora_ids, ora_vals, gpu_true, rel_tie=REL_TIE, rel_dist=REL_DIST) -> dict:
    """Counts of the rule's violations. ``gpu_true``: the oracle's exact values of the GPU's ids at
    the GPU's positions (NaN = unknown, never a tie)."""
    gpu_ids = np.asarray(gpu_ids).view(np.uint32)
    ora_ids = np.asarray(ora_ids).view(np.uint32)
    valid = ora_ids != INVALID
    scale = np.maximum(np.abs(np.where(valid, ora_vals, 1.0)), 1e-6)
    dist_err = np.where(valid, np.abs(np.where(valid, gpu_vals, 0) - np.where(valid, ora_vals, 0)) / scale, 0)
    mism = (gpu_ids != ora_ids) & valid
    tie_err = np.abs(np.nan_to_num(np.asarray(gpu_true, np.float64), nan=np.inf) - ora_vals) / scale
    bad = mism & ~(tie_err <= rel_tie)
    dups = sum(len(np.unique(r[r != INVALID])) != int((r != INVALID).sum()) for r in gpu_ids)
    return {"queries": int(gpu_ids.shape[0]), "k": int(gpu_ids.shape[1]),
            "id_mismatches_outside_ties": int(bad.sum()), "id_mismatches_within_ties": int((mism & ~bad).sum()),
            "max_rel_dist_err": float(dist_err[valid].max()) if valid.any() else 0.0,
            "dist_within_tol": bool(np.all(dist_err[valid] <= rel_dist)),
            "padding_matches": bool(np.array_equal(gpu_ids == INVALID, ora_ids == INVALID)),
            "rows_with_duplicate_ids": int(dups),
            "rule": "ids bit-exact except ties within 1e-5 relative; distances within 1e-4 relative"}


def ok(s: dict) -> bool:
    return (s["id_mismatches_outside_ties"] == 0 and s["dist_within_tol"] and s["padding_matches"]
            and s["rows_with_duplicate_ids"] == 0)
