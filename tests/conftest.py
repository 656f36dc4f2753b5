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
    """Parity rule of the project brief (oracle/parity.py): returned ids bit-exact except where
    distances tie within ``rel_tie`` relative; distances within ``rel_dist`` relative of the oracle's.

    ``gpu_true_vals`` are the oracle's exact values for the ids the GPU returned (same positions).
    """
    from oracle import parity
    gpu_ids = np.asarray(gpu_ids)
    ora_ids = np.asarray(ora_ids)
    assert gpu_ids.shape == ora_ids.shape
    s = parity.summary(gpu_ids, gpu_vals, ora_ids, ora_vals, gpu_true_vals, rel_tie, rel_dist)
    assert parity.ok(s), f"parity rule violated: {s}"
    valid = ora_ids.view(np.uint32) != 0xFFFFFFFF
    mism = (gpu_ids.view(np.uint32) != ora_ids.view(np.uint32)) & valid
    return float(1.0 - mism.sum() / max(1, valid.sum()))
