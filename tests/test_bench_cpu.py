"""The measurement harness's CPU-side contract (no GPU): the reference arm's JSON line, the
cross-rank merge the parity check uses, and the AUTO precision mirror.

The reference arm (`bench.py --impl reference`) times the CPU restatement of the reference's
search path on the host cores; its line must carry the same metric and config as the GPU arm
(the driver compares them) plus `impl`, `cpu_baseline` and `e2e`."""

import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _bench():
    import bench
    return bench


def test_reference_arm_prints_the_contract_line():
    args = ["--impl", "reference", "--n", "20000", "--nq", "40", "--steps", "1", "--warmup", "0",
            "--cpu-rows", "20000"]
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference" and line["unit"] == "queries/s" and line["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    # the same metric and config dict as the GPU arm's line for these arguments
    b = _bench()
    saved = sys.argv
    try:
        sys.argv = ["bench.py", *args]
        a = b.parse_args()
    finally:
        sys.argv = saved
    assert line["metric"] == b.METRIC
    assert line["config"] == b.workload(a)


def _merge_ref(va, ia, vb, ib, k, larger):
    rows = []
    for r in range(va.shape[0]):
        c = [(v, i) for v, i in zip(np.r_[va[r], vb[r]], np.r_[ia[r], ib[r]]) if i != 0xFFFFFFFF]
        c.sort(key=lambda t: ((-t[0] if larger else t[0]), t[1]))
        rows.append(c[:k])
    return rows


@pytest.mark.parametrize("larger", [False, True])
def test_merge_best_orders_by_value_then_id(larger):
    b = _bench()
    rng = np.random.default_rng(3)
    va = rng.integers(0, 5, (50, 8)).astype(np.float32)  # many equal values: the id decides
    vb = rng.integers(0, 5, (50, 8)).astype(np.float32)
    ia = rng.choice(1000, (50, 8)).astype(np.uint32)
    ib = (rng.choice(1000, (50, 8)) + 1000).astype(np.uint32)
    ia[:, -1] = 0xFFFFFFFF  # padding never wins
    v, i = b.merge_best(va, ia, vb, ib, 6, larger)
    ref = _merge_ref(va, ia, vb, ib, 6, larger)
    for r in range(50):
        assert [(float(x), int(y)) for x, y in zip(v[r], i[r])] == [(float(x), int(y)) for x, y in ref[r]]


@pytest.mark.parametrize("k,rerank,f32,want", [(10, 0, True, "bf16"), (100, 0, True, "bf16"),
                                               (10, 4, True, "bf16"), (10, 2, True, "bf16"), (50, 2, True, "tf32"),
                                               (100, 1, False, "tf32")])
def test_auto_precision_mirrors_the_library_rule(k, rerank, f32, want):
    # AUTO: bf16 when the pool holds >= 3k candidates (fp32 rows without a caller's factor widen
    # the pool to 3k), else tf32 (plan_route in va_search.cu)
    assert _bench().auto_precision(k, rerank, f32) == want
