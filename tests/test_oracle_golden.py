"""The CPU oracle against the reference's own known answers (tests/golden/known_answers.json,
transcribed from VectorAccelerate's XCTest suite). CPU only."""

import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "known_answers.json")


def _cases(kind):
    with open(GOLDEN) as f:
        return [c for c in json.load(f)["cases"] if c["kind"] == kind]


def _f(v):
    return np.array([[float("inf") if x == "inf" else x for x in row] for row in v], np.float32)


@pytest.mark.parametrize("case", _cases("knn"), ids=lambda c: c["source"])
def test_oracle_knn_known_answers(oracle, case):
    ids, vals = oracle.knn(np.array(case["queries"], np.float32), np.array(case["database"], np.float32), case["k"])
    assert ids.tolist() == case["ids"]
    np.testing.assert_allclose(vals, _f(case["values"]), atol=case["tol"])


@pytest.mark.parametrize("case", _cases("topk"), ids=lambda c: c["source"])
def test_oracle_topk_known_answers(oracle, case):
    vals, ids = oracle.topk_select(np.array(case["values_in"], np.float32), case["k"], 1 if case["mode"] == "max" else 0)
    assert ids.tolist() == case["ids"]
    np.testing.assert_allclose(vals, _f(case["values"]), atol=case["tol"])


@pytest.mark.parametrize("case", _cases("hamming_pairs"), ids=lambda c: c["source"])
def test_oracle_hamming_known_answers(oracle, case):
    codes = oracle.binary_quantize(np.array(case["vectors"], np.float32))
    m = oracle.hamming_matrix(codes[case["query"]:case["query"] + 1], codes)
    assert m[0].tolist() == case["distances"]


@pytest.mark.parametrize("case", _cases("hamming_matrix"), ids=lambda c: c["source"])
def test_oracle_hamming_matrix(oracle, case):
    q = oracle.binary_quantize(np.array(case["queries_bits"], np.float32))
    x = oracle.binary_quantize(np.array(case["database_bits"], np.float32))
    assert oracle.hamming_matrix(q, x)[0].tolist() == case["row0"]


@pytest.mark.parametrize("case", _cases("pack_bits"), ids=lambda c: c["source"])
def test_oracle_pack_bits(oracle, case):
    bits = np.array(case["bits"], np.float32)[None, :]
    assert oracle.binary_quantize(bits)[0].tolist() == case["words"]


@pytest.mark.parametrize("case", _cases("sq_roundtrip"), ids=lambda c: c["source"])
def test_oracle_sq_roundtrip(oracle, case):
    x = np.array(case["data"], np.float32)
    scale, zp = oracle.sq_params(x, 0, case["bits"])
    if case["bits"] == 8:
        rec = oracle.dequantize_int8(oracle.quantize_int8(x, scale, zp), scale, zp)
    else:
        rec = oracle.dequantize_int4(oracle.quantize_int4(x, scale, zp), x.size, scale, zp)
    np.testing.assert_allclose(rec, x, atol=case["tol"])


@pytest.mark.parametrize("case", _cases("sq_order"), ids=lambda c: c["source"])
def test_oracle_sq_order(oracle, case):
    x = np.array(case["data"], np.float32)
    scale, zp = oracle.sq_params(x, 0, 8)
    rec = oracle.dequantize_int8(oracle.quantize_int8(x, scale, zp), scale, zp)
    assert np.all(np.diff(rec) > 0)


def test_oracle_asymmetric_params(oracle):
    # KernelTests.swift:1790-1802 quantizes [0, 0.1, ..., 0.5] both ways. Asymmetric parameters
    # (ScalarQuantizationKernel.swift:512-518): scale = range / 255, zero point
    # Int8(clamping: -round(min / scale)) = 0 for min = 0; symmetric: scale = absmax / 127, zp 0.
    x = np.array([0.0, 0.1, 0.2, 0.3, 0.4, 0.5], np.float32)
    ss, zs = oracle.sq_params(x, 0, 8)
    sa, za = oracle.sq_params(x, 1, 8)
    assert zs == 0 and za == 0
    assert ss == pytest.approx(0.5 / 127, rel=1e-6)
    assert sa == pytest.approx(0.5 / 255, rel=1e-6)
    # A negative minimum gives a positive zero point, saturating at 127.
    sa2, za2 = oracle.sq_params(np.array([-1.0, 0.5], np.float32), 1, 8)
    assert za2 == 127  # -round(-1 / (1.5/255)) = 170 -> clamped


def test_oracle_tie_rule(oracle):
    # Equal distances keep the smaller id (AdvancedTopK.metal:48-52).
    q = np.zeros((1, 2), np.float32)
    x = np.array([[1, 0], [0, 1], [-1, 0], [0, -1], [2, 0]], np.float32)
    ids, vals = oracle.knn(q, x, 3)
    assert ids.tolist() == [[0, 1, 2]]
    # inner products with [1, 0]: 1, 0, -1, 0, 2 -> 4, 0, then the tie 1 / 3 keeps 1
    ids, vals = oracle.knn(np.array([[1, 0]], np.float32), x, 3, metric=oracle.METRIC_IP)
    assert ids.tolist() == [[4, 0, 1]]
    assert vals.tolist() == [[2.0, 1.0, 0.0]]


def test_oracle_rng_is_testrng(oracle):
    # TestRNG.swift:57-104: seed 0 behaves like seed 1 and streams differ.
    a = oracle.gen_gaussian(2, 8, 0)
    b = oracle.gen_gaussian(2, 8, 1)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a[0], a[1])
    g = oracle.gen_gaussian(20000, 64, 7)
    assert abs(float(g.mean())) < 0.01 and abs(float(g.std()) - 1.0) < 0.01


def test_oracle_fp32_mode_matches_truth(oracle):
    x = oracle.gen_gaussian(3000, 96, 0)
    q = oracle.gen_gaussian(20, 96, 1, row0=1 << 31)
    i32, v32 = oracle.knn(q, x, 10, truth=False)
    i64, v64 = oracle.knn(q, x, 10, truth=True)
    np.testing.assert_allclose(v32, v64, rtol=1e-5)


def test_oracle_int8_pipeline(oracle):
    x = oracle.gen_mixture(2000, 64, 0, 16, 0.3, False)
    q = oracle.gen_mixture(8, 64, 5, 16, 0.3, False)
    mins, scales = oracle.sq_perdim_params(x)
    xc = oracle.sq_perdim_quantize(x, mins, scales)
    qc = oracle.sq_perdim_quantize(q, mins, scales)
    ids, vals, cids, cd = oracle.int8_knn(qc, q, xc, x, 100, 10)
    tids, tvals = oracle.knn(q, x, 10)
    # the integer pass keeps the true neighbours in its 100-candidate pool on this data
    assert (ids == tids).mean() > 0.95
    assert np.all(np.diff(cd, axis=1) >= 0)

