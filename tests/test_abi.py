"""The C ABI boundary without a GPU: the library loads, exports every function declared in
include/va_cuda.h, and the host mirror validates parameters like the reference
(FusedL2TopKKernel.swift:52-85, checked by KernelTests.swift:939-1046)."""

import ctypes
import json
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "va_cuda.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(va_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = _declared()
    for required in ("va_context_create", "va_knn_search", "va_knn_search_host", "va_topk_select",
                     "va_topk_merge", "va_merge_shards", "va_l2_distance_pairs", "va_cosine_pairs",
                     "va_distance_matrix", "va_sq_quantize_int8", "va_binary_quantize", "va_hamming_knn",
                     "va_hamming_matrix", "va_db_create", "va_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from vectoraccelerate_b200 import _ffi
    lib = _ffi.load()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    # and the ctypes signature table covers every declaration
    assert not [n for n in _declared() if n not in _ffi.SIGNATURES]


def test_library_has_no_cuda_runtime_dependency():
    # the runtime is linked statically; the library must load on a host without the toolkit
    import subprocess
    out = subprocess.run(["ldd", os.path.join(ROOT, "vectoraccelerate_b200", "libva_cuda.so")],
                         capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


def test_abi_version():
    from vectoraccelerate_b200 import _ffi
    assert _ffi.load().va_abi_version() == 1


def test_calls_fail_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import vectoraccelerate_b200 as va
    with pytest.raises(va.ComputeFailed):
        va.GPUContext()


def test_null_arguments_are_rejected():
    from vectoraccelerate_b200 import _ffi
    lib = _ffi.load()
    assert lib.va_context_create(None, None) == -1
    assert "out must not be NULL" in _ffi.last_error()
    assert lib.va_topk_select(None, None, 1, 1, 1, 1, 0, None, None, 1) == -1
    assert lib.va_knn_search(None, None, None, 1, 1, 0, 0, 0, None, None) == -1


def _golden(kind):
    with open(os.path.join(ROOT, "tests", "golden", "known_answers.json")) as f:
        return [c for c in json.load(f)["cases"] if c["kind"] == kind]


@pytest.mark.parametrize("case", _golden("validate"), ids=lambda c: json.dumps(c["params"]))
def test_fused_parameter_validation_messages(case):
    import vectoraccelerate_b200 as va
    P = va.FusedL2TopKParameters
    p = dict(case["params"])
    if p["dimension"] == "maxDimension+1":
        p["dimension"] = P.maxDimension + 1
    if p["k"] == "maxK+1":
        p["k"] = P.maxK + 1
    with pytest.raises(va.errors.IndexError) as ei:
        P(p["numQueries"], p["numDataset"], p["dimension"], p["k"])
    msg = str(ei.value)
    for word in case["message_contains"]:
        word = {"maxDimension": str(P.maxDimension), "maxK": str(P.maxK)}.get(word, word)
        assert word in msg


def test_fused_parameter_validation_success():
    import vectoraccelerate_b200 as va
    va.FusedL2TopKParameters(1, 100, 768, 8)
    va.FusedL2TopKParameters(10, 10_000, va.FusedL2TopKParameters.maxDimension, va.FusedL2TopKParameters.maxK)


def test_pack_binary_host_helper():
    import vectoraccelerate_b200 as va
    assert va.HammingDistanceKernel.pack_binary([1, 0, 1, 0, 0, 0, 0, 0]).tolist() == [5]
    assert va.HammingDistanceKernel.pack_binary([1] * 64).tolist() == [0xFFFFFFFF, 0xFFFFFFFF]


def test_binary_vector_helpers():
    import vectoraccelerate_b200 as va
    a = va.Metal4BinaryVector(np.array([0b1100], np.uint32), 4)
    b = va.Metal4BinaryVector(np.array([0b1010], np.uint32), 4)
    assert a.hamming_distance(b) == 2 and a.bit(2) and not a.bit(0) and not a.bit(9)


def test_nccl_unique_id_without_a_gpu():
    # NCCL is loaded at run time; making a unique id needs no GPU
    import vectoraccelerate_b200 as va
    a, b = va.nccl_unique_id(), va.nccl_unique_id()
    assert len(a) == 128 and a != b
