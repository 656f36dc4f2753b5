import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libva_cuda.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def ctx():
    import vectoraccelerate_b200 as va
    c = va.GPUContext()
    yield c
    c.close()


def assert_knn_parity(gpu_ids, gpu_vals, ora_ids, ora_vals, gpu_true_vals, rel_tie=1e-5, rel_dist=1e-4,
                      larger_is_better=False):
    """Parity rule of the project brief: returned ids bit-exact except where distances tie within
    ``rel_tie`` relative; distances within ``rel_dist`` relative of the oracle's.

    ``gpu_true_vals`` are the oracle's exact values for the ids the GPU returned (same positions).
    """
    gpu_ids = np.asarray(gpu_ids)
    ora_ids = np.asarray(ora_ids)
    assert gpu_ids.shape == ora_ids.shape
    valid = ora_ids != 0xFFFFFFFF
    scale = np.maximum(np.abs(np.where(valid, ora_vals, 1.0)), 1e-6)
    dist_err = np.where(valid, np.abs(np.where(valid, gpu_vals, 0) - np.where(valid, ora_vals, 0)), 0) / scale
    assert np.all(dist_err[valid] <= rel_dist), f"max relative distance error {dist_err[valid].max():.3g}"
    assert np.array_equal(gpu_ids == 0xFFFFFFFF, ora_ids == 0xFFFFFFFF), "padding differs"
    mism = (gpu_ids != ora_ids) & valid
    if mism.any():
        tie_err = np.abs(gpu_true_vals - ora_vals) / scale
        bad = mism & (tie_err > rel_tie)
        assert not bad.any(), (
            f"{int(bad.sum())} id mismatches outside ties; first at {np.argwhere(bad)[0]}: "
            f"gpu id {gpu_ids[bad][0]} (true {gpu_true_vals[bad][0]!r}) vs oracle id {ora_ids[bad][0]} "
            f"({ora_vals[bad][0]!r})")
    for r in range(gpu_ids.shape[0]):
        v = gpu_ids[r][gpu_ids[r] != 0xFFFFFFFF]
        assert len(np.unique(v)) == len(v), f"duplicate ids in row {r}"
    return float(1.0 - mism.sum() / max(1, valid.sum()))
