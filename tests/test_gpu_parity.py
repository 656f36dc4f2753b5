"""GPU parity: every libva_cuda entry point against the CPU oracle on identical seeded inputs,
plus the reference's known answers through the C ABI. Needs a B200."""

import json
import os

import numpy as np
import pytest

from conftest import assert_knn_parity

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
QROW = 1 << 31  # query streams are offset from database streams (TestRNG maps seed 0 to seed 1)


def _golden(kind):
    with open(os.path.join(ROOT, "tests", "golden", "known_answers.json")) as f:
        return [c for c in json.load(f)["cases"] if c["kind"] == kind]


def _f(v):
    return np.array([[float("inf") if x == "inf" else x for x in row] for row in v], np.float32)


def _knn(ctx, x, q, k, metric=0, precision=0, rerank=0, dtype=0, id_base=0):
    import vectoraccelerate_b200 as va
    db = va.Database(ctx, x, dtype=dtype, id_base=id_base)
    try:
        return va.knn_search_host(ctx, db, q, k, metric, precision, rerank)
    finally:
        db.close()


def _check(oracle, q, x, k, metric, vals, ids, db_bf16=False):
    tids, tvals = oracle.knn(q, x, k, metric=metric, db_bf16=db_bf16)
    gtrue_ids, gtrue = oracle.rerank(q, x, ids, k, metric=metric, db_bf16=db_bf16)
    # true values of the GPU's ids at the GPU's positions
    gt = np.full(ids.shape, np.inf if metric != 2 else -np.inf, np.float32)
    for r in range(ids.shape[0]):
        pos = {int(i): j for j, i in enumerate(gtrue_ids[r])}
        for j, i in enumerate(ids[r]):
            if int(i) in pos:
                gt[r, j] = gtrue[r, pos[int(i)]]
    return assert_knn_parity(ids, vals, tids, tvals, gt)


# ------------------------------------------------------------------------------------------------ known answers
@pytest.mark.parametrize("case", _golden("knn"), ids=lambda c: c["source"])
@pytest.mark.parametrize("precision", [1, 2, 3])
def test_knn_known_answers(ctx, case, precision):
    vals, ids = _knn(ctx, np.array(case["database"], np.float32), np.array(case["queries"], np.float32),
                     case["k"], precision=precision)
    assert ids.tolist() == case["ids"]
    np.testing.assert_allclose(vals, _f(case["values"]), atol=case["tol"])


def test_fused_kernel_known_answer(ctx):
    import vectoraccelerate_b200 as va
    kern = va.FusedL2TopKKernel(ctx)
    res = kern.find_nearest_neighbors([[0, 0, 0, 0]], [[1, 0, 0, 0], [2, 0, 0, 0], [0.5, 0, 0, 0], [3, 0, 0, 0]], 2)
    assert [r[0] for r in res[0]] == [2, 0]
    assert res[0][0][1] == pytest.approx(0.25, abs=1e-4) and res[0][1][1] == pytest.approx(1.0, abs=1e-4)


@pytest.mark.parametrize("case", _golden("topk"), ids=lambda c: c["source"])
def test_topk_known_answers(ctx, case):
    import vectoraccelerate_b200 as va
    vals, ids = va.TopKSelectionKernel(ctx).select_arrays(np.array(case["values_in"], np.float32), case["k"],
                                                         "maximum" if case["mode"] == "max" else "minimum")
    assert ids.tolist() == case["ids"]
    np.testing.assert_allclose(vals, _f(case["values"]), atol=case["tol"])


@pytest.mark.parametrize("case", _golden("hamming_pairs"), ids=lambda c: c["source"])
def test_hamming_known_answers(ctx, case):
    import vectoraccelerate_b200 as va
    bq = va.BinaryQuantizationKernel(ctx)
    vecs = bq.quantize(np.array(case["vectors"], np.float32))
    d = bq.compute_hamming_distances(vecs[case["query"]], vecs)
    assert d.tolist() == [float(v) for v in case["distances"]]


@pytest.mark.parametrize("case", _golden("hamming_matrix"), ids=lambda c: c["source"])
def test_hamming_matrix_known_answer(ctx, case):
    import vectoraccelerate_b200 as va
    m = va.HammingDistanceKernel(ctx).distance_matrix([[bool(b) for b in r] for r in case["queries_bits"]],
                                                      [[bool(b) for b in r] for r in case["database_bits"]])
    assert m[0].tolist() == [float(v) for v in case["row0"]]


@pytest.mark.parametrize("case", _golden("sq_roundtrip"), ids=lambda c: c["source"])
def test_sq_roundtrip_known_answers(ctx, case):
    import vectoraccelerate_b200 as va
    k = va.ScalarQuantizationKernel(ctx)
    x = np.array(case["data"], np.float32)
    r = k.quantize(x, bit_width=case["bits"])
    np.testing.assert_allclose(k.dequantize(r, x.size), x, atol=case["tol"])


# ------------------------------------------------------------------------------------------------ generation
def test_device_generator_matches_oracle(ctx, oracle):
    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi
    rows, dim = 257, 96
    buf = ctx.get_buffer(rows * dim * 4, np.float32, (rows, dim))
    _ffi.call("va_gen_gaussian", ctx.handle, buf.ptr, rows, dim, 3, 1000)
    g = buf.download()
    o = oracle.gen_gaussian(rows, dim, 3, row0=1000)
    ulps = np.abs(g.view(np.int32).astype(np.int64) - o.view(np.int32).astype(np.int64))
    assert (ulps > 1).sum() == 0 and (ulps == 1).mean() < 1e-3
    _ffi.call("va_gen_mixture", ctx.handle, buf.ptr, rows, dim, 5, 0, 16, 0.3, 1)
    g = buf.download()
    o = oracle.gen_mixture(rows, dim, 5, 16, 0.3, True)
    np.testing.assert_allclose(g, o, rtol=0, atol=2e-7)


# ------------------------------------------------------------------------------------------------ distances
def test_l2_and_cosine_pairs(ctx, oracle):
    import vectoraccelerate_b200 as va
    a = oracle.gen_gaussian(333, 77, 1)
    b = oracle.gen_gaussian(333, 77, 2)
    for sq in (False, True):
        np.testing.assert_allclose(va.L2DistanceKernel(ctx).compute_pairs(a, b, sq), oracle.l2_pairs(a, b, sq),
                                   rtol=1e-5)
    for dist in (False, True):
        np.testing.assert_allclose(va.CosineSimilarityKernel(ctx).compute_pairs(a, b, dist),
                                   oracle.cosine_pairs(a, b, dist), rtol=1e-5, atol=1e-6)
    z = np.zeros((2, 77), np.float32)
    assert va.CosineSimilarityKernel(ctx).compute_pairs(z, a[:2]).tolist() == [0.0, 0.0]


@pytest.mark.parametrize("metric,flag", [(0, False), (0, True), (1, False), (1, True), (2, False), (2, True)])
def test_distance_matrix(ctx, oracle, metric, flag):
    from vectoraccelerate_b200 import kernels
    q = oracle.gen_gaussian(70, 100, 1)
    x = oracle.gen_gaussian(131, 100, 2)
    g = kernels._matrix(ctx, q, x, metric, flag)
    o = oracle.matrix(q, x, metric, flag)
    np.testing.assert_allclose(g, o, rtol=1e-4, atol=1e-4)


# ------------------------------------------------------------------------------------------------ selection
@pytest.mark.parametrize("k", [1, 8, 9, 32, 33, 100, 128, 1000])
@pytest.mark.parametrize("mode", ["minimum", "maximum"])
def test_topk_select_random(ctx, oracle, k, mode):
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(k)
    v = rng.standard_normal((37, 5000)).astype(np.float32)
    vals, ids = va.TopKSelectionKernel(ctx).select_arrays(v, k, mode)
    ov, oi = oracle.topk_select(v, k, 1 if mode == "maximum" else 0)
    assert np.array_equal(ids, oi) and np.array_equal(vals, ov)


def test_topk_select_ties_and_padding(ctx, oracle):
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(0)
    v = rng.integers(0, 5, (20, 3000)).astype(np.float32)  # massive ties: smaller index wins
    for mode in ("minimum", "maximum"):
        vals, ids = va.TopKSelectionKernel(ctx).select_arrays(v, 64, mode)
        ov, oi = oracle.topk_select(v, 64, 1 if mode == "maximum" else 0)
        assert np.array_equal(ids, oi)
    vals, ids = va.TopKSelectionKernel(ctx).select_arrays(v[:, :5], 9)
    assert (ids[:, 5:] == 0xFFFFFFFF).all() and np.isinf(vals[:, 5:]).all()


def test_topk_merge(ctx, oracle):
    import vectoraccelerate_b200 as va
    rng = np.random.default_rng(1)
    rv = np.sort(rng.random((16, 10)).astype(np.float32), axis=1)
    ri = rng.permutation(1000)[:160].reshape(16, 10).astype(np.uint32)
    cv = np.sort(rng.random((16, 7)).astype(np.float32), axis=1)
    ci = np.tile(np.arange(7, dtype=np.uint32), (16, 1))
    gv, gi = va.TopKMergeKernel(ctx).merge(rv, ri, cv, ci, 5000)
    ov, oi = oracle.topk_merge(rv, ri, cv, ci, 5000)
    assert np.array_equal(gi, oi) and np.array_equal(gv, ov)


# ------------------------------------------------------------------------------------------------ fused search
@pytest.fixture(scope="module")
def c1(oracle):
    """Config 1 of the benchmark brief: N=10,000 x 768 N(0,1) seed 0; 1,000 queries seed 1; k=10."""
    x = oracle.gen_gaussian(10_000, 768, 0)
    q = oracle.gen_gaussian(1_000, 768, 1, row0=QROW)
    ids, vals = oracle.knn(q, x, 10)
    return x, q, ids, vals


@pytest.mark.parametrize("precision", [1, 2, 3], ids=["fp32", "tf32", "bf16"])
def test_c1_full_parity(ctx, oracle, c1, precision):
    x, q, tids, tvals = c1
    vals, ids = _knn(ctx, x, q, 10, precision=precision)
    frac = _check(oracle, q, x, 10, 0, vals, ids)
    assert frac >= 0.999


@pytest.mark.parametrize("metric", [0, 1, 2], ids=["l2", "cosine", "ip"])
@pytest.mark.parametrize("shape", [(1, 1, 4, 3), (3, 257, 100, 10), (129, 3001, 64, 1), (200, 2000, 130, 21),
                                   (1, 600, 768, 16), (300, 5000, 33, 5)],
                         ids=lambda s: "q{}-n{}-d{}-k{}".format(*s))
def test_fused_shapes(ctx, oracle, metric, shape):
    nq, n, d, k = shape
    x = oracle.gen_mixture(n, d, 11, 8, 0.3, metric == 1)
    q = oracle.gen_mixture(nq, d, 12, 8, 0.3, metric == 1)
    for precision in (1, 3):
        vals, ids = _knn(ctx, x, q, k, metric=metric, precision=precision)
        _check(oracle, q, x, k, metric, vals, ids)


def test_fused_bf16_database(ctx, oracle):
    x32 = oracle.gen_mixture(4000, 256, 3, 32, 0.25, True)
    xb = oracle.f32_to_bf16(x32)
    q = oracle.gen_mixture(64, 256, 4, 32, 0.25, True)
    vals, ids = _knn(ctx, xb, q, 10, metric=2, dtype=1)
    _check(oracle, q, xb, 10, 2, vals, ids, db_bf16=True)


def test_fused_ties_keep_smaller_id(ctx, oracle):
    # duplicated rows give exact distance ties: ids must come out in increasing order
    base = oracle.gen_gaussian(50, 64, 9)
    x = np.concatenate([base] * 6)
    q = oracle.gen_gaussian(7, 64, 10)
    for precision in (1, 2, 3):
        vals, ids = _knn(ctx, x, q, 12, precision=precision)
        tids, tvals = oracle.knn(q, x, 12)
        assert np.array_equal(ids, tids)


def test_sharded_merge_equals_single(ctx, oracle):
    import vectoraccelerate_b200 as va
    from vectoraccelerate_b200 import _ffi
    x = oracle.gen_gaussian(6000, 96, 21)
    q = oracle.gen_gaussian(50, 96, 22, row0=QROW)
    k, parts = 10, []
    bounds = [0, 1000, 2500, 4000, 6000]
    for s in range(4):
        parts.append(_knn(ctx, x[bounds[s]:bounds[s + 1]], q, k, id_base=bounds[s]))
    gv = np.stack([p[0] for p in parts])
    gi = np.stack([p[1] for p in parts])
    dv, di = ctx.get_buffer_for(gv), ctx.get_buffer_for(gi)
    ov = ctx.get_buffer(4 * 50 * k, np.float32, (50, k))
    oi = ctx.get_buffer(4 * 50 * k, np.uint32, (50, k))
    _ffi.call("va_merge_shards", ctx.handle, dv.ptr, di.ptr, 4, 50, k, 0, ov.ptr, oi.ptr)
    tids, tvals = oracle.knn(q, x, k)
    assert np.array_equal(oi.download(), tids)


def test_invalid_search_arguments(ctx):
    import vectoraccelerate_b200 as va
    x = np.zeros((10, 8), np.float32)
    db = va.Database(ctx, x)
    with pytest.raises(va.InvalidInput, match="k 2000 exceeds maximum supported k 1024"):
        va.knn_search_host(ctx, db, np.zeros((1, 8), np.float32), 2000)
    with pytest.raises(va.InvalidInput, match="dimension"):
        va.knn_search_host(ctx, db, np.zeros((1, 9), np.float32), 3)
    with pytest.raises(va.InvalidInput, match="dimension 5000 exceeds maximum supported dimension 4096"):
        va.Database(ctx, np.zeros((2, 5000), np.float32))
    db.close()


# ------------------------------------------------------------------------------------------------ index
def test_index_search_known_values_and_deletion(ctx):
    import vectoraccelerate_b200 as va
    idx = va.AcceleratedVectorIndex(va.IndexConfiguration.flat(4), ctx)
    h = idx.insert([3, 4, 0, 0])
    r = idx.search([0, 0, 0, 0], 1)
    assert r.count == 1 and r.results[0].distance == pytest.approx(25.0, abs=1e-3) and r.results[0].id == h
    h2 = idx.insert([1, 2, 3, 4])
    h3 = idx.insert([0.1, 0, 0, 0])
    r = idx.search([0, 0, 0, 0], 2)
    assert [x.id for x in r.results] == [h3, h]
    idx.remove(h3)
    r = idx.search([0, 0, 0, 0], 2)
    assert [x.id for x in r.results] == [h, h2]
    assert [x.distance for x in r.results] == pytest.approx([25.0, 30.0])
    batch = idx.search_batch(np.array([[0, 0, 0, 0], [1, 2, 3, 4]], np.float32), 1)
    assert batch[1].results[0].id == h2 and batch[1].results[0].distance == 0.0


# ------------------------------------------------------------------------------------------------ quantization
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("type_", ["symmetric", "asymmetric"])
def test_sq_bit_exact(ctx, oracle, bits, type_):
    import vectoraccelerate_b200 as va
    x = (oracle.gen_gaussian(1, 10001, 4)[0] * 3).astype(np.float32)
    k = va.ScalarQuantizationKernel(ctx)
    r = k.quantize(x, bit_width=bits, type=type_)
    scale, zp = oracle.sq_params(x, 1 if type_ == "asymmetric" else 0, bits)
    assert r.scale == pytest.approx(scale, rel=0) and (r.zero_point or 0) == zp
    if bits == 8:
        ref = oracle.quantize_int8(x, scale, zp)
        assert np.array_equal(np.frombuffer(r.quantized_data, np.int8), ref)
        np.testing.assert_array_equal(k.dequantize(r, x.size), oracle.dequantize_int8(ref, scale, zp))
    else:
        ref = oracle.quantize_int4(x, scale, zp)
        assert np.array_equal(np.frombuffer(r.quantized_data, np.uint8), ref)
        np.testing.assert_array_equal(k.dequantize(r, x.size), oracle.dequantize_int4(ref, x.size, scale, zp))


def test_sq_per_channel(ctx, oracle):
    from vectoraccelerate_b200 import _ffi
    x = oracle.gen_gaussian(1, 4000, 5)[0]
    scales = np.array([0.01, 0.02, 0.03, 0.04], np.float32)
    zps = np.array([0, 3, -2, 7], np.int8)
    dx, ds, dz = ctx.get_buffer_for(x), ctx.get_buffer_for(scales), ctx.get_buffer_for(zps)
    out = ctx.get_buffer(x.size, np.int8, (x.size,))
    _ffi.call("va_sq_quantize_int8", ctx.handle, dx.ptr, x.size, 1.0, 0, ds.ptr, dz.ptr, 4, out.ptr)
    assert np.array_equal(out.download(), oracle.quantize_int8(x, 1.0, 0, scales, zps, 4))


# ------------------------------------------------------------------------------------------------ binary / Hamming
def test_binary_quantize_and_hamming(ctx, oracle):
    import vectoraccelerate_b200 as va
    for d in (4, 32, 100, 1024):
        x = oracle.gen_gaussian(301, d, d)
        codes = va.BinaryQuantizationKernel(ctx).quantize_array(x)
        assert np.array_equal(codes, oracle.binary_quantize(x))
    q = codes[:17]
    m = va.HammingDistanceKernel(ctx).compute_bit_packed(q, codes, 1024)
    assert np.array_equal(m, oracle.hamming_matrix(q, codes))


@pytest.mark.parametrize("words,k", [(32, 100), (32, 1), (4, 10), (1, 16), (2, 7), (8, 128)])
def test_hamming_knn(ctx, oracle, words, k):
    import vectoraccelerate_b200 as va
    n = 20_000
    x = oracle.binary_quantize(oracle.gen_gaussian(n, words * 32, 2))
    q = oracle.binary_quantize(oracle.gen_gaussian(300, words * 32, 3, row0=QROW))
    gd, gi = va.HammingDistanceKernel(ctx).nearest_neighbors(q, x, k)
    oi, od = oracle.hamming_knn(q, x, k)
    assert np.array_equal(gd, od)
    assert np.array_equal(gi, oi)  # integer distances: (distance, id) order is exact


def test_pair_kernel_parity(oracle, c1, tmp_path):
    """The cta_group::2 pair kernel (selected per process by VA_TC_PAIR=1) on the C1 workload."""
    import subprocess
    import sys
    x, q, tids, tvals = c1
    np.save(tmp_path / "x.npy", x)
    np.save(tmp_path / "q.npy", q)
    code = (
        "import sys, numpy as np; sys.path.insert(0, %r)\n"
        "import vectoraccelerate_b200 as va\n"
        "x = np.load(%r); q = np.load(%r)\n"
        "ctx = va.GPUContext(); db = va.Database(ctx, x)\n"
        "for m in (0, 2):\n"
        "    v, i = va.knn_search_host(ctx, db, q, 10, m, va.PREC_BF16)\n"
        "    np.save(%r %% m, v); np.save(%r %% m, i)\n"
    ) % (ROOT, str(tmp_path / "x.npy"), str(tmp_path / "q.npy"), str(tmp_path / "v%d.npy"),
         str(tmp_path / "i%d.npy"))
    env = dict(os.environ, VA_TC_PAIR="1")
    subprocess.run([sys.executable, "-c", code], check=True, env=env, timeout=600)
    for metric in (0, 2):
        vals = np.load(tmp_path / f"v{metric}.npy")
        ids = np.load(tmp_path / f"i{metric}.npy")
        frac = _check(oracle, q, x, 10, metric, vals, ids)
        assert frac >= 0.999


@pytest.mark.parametrize("metric,n,d,k,prec", [(1, 30_000, 1536, 100, 0), (0, 40_000, 768, 50, 0),
                                               (2, 25_000, 256, 100, 0), (0, 20_000, 128, 42, 0),
                                               (1, 30_000, 1536, 100, 2), (2, 25_000, 256, 100, 2)],
                         ids=["cos-k100-d1536", "l2-k50", "ip-k100", "l2-k42", "cos-k100-tf32", "ip-k100-tf32"])
def test_fused_large_k(ctx, oracle, metric, n, d, k, prec):
    """Large k on the tensor-core route. Auto precision over fp32 rows: bf16 with a 3k pool
    (wider than the 128-entry lists from k = 43 on); explicit TF32: the k + max(k/4, 22) pool."""
    x = oracle.gen_mixture(n, d, 31, 64, 0.3, metric == 1)
    q = oracle.gen_mixture(96, d, 32, 64, 0.3, metric == 1)
    vals, ids = _knn(ctx, x, q, k, metric=metric, precision=prec)
    frac = _check(oracle, q, x, k, metric, vals, ids)
    assert frac >= 0.999
