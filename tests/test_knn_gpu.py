"""GPU parity of the flat kNN path against the CPU oracle, through the C ABI.

The bar: neighbour ids identical to the oracle's (score, id) order and
distances bit-identical (the GPU re-ranks in the reference's AVX-512
arithmetic order); Minkowski distances within 1e-6 relative (the cube root
is CUDA's cbrtf, the oracle's is glibc's; ranking uses the pre-root sum on
both sides). Cases mirror the reference's tests
(crates/vector-cuda/src/knn.rs:404-542,
crates/vector-cuda/tests/integration_tests.rs) plus seeded random shapes.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


def _engine(vc, base, metric, g=1, mode=0):
    base = np.ascontiguousarray(base, np.float32)
    return vc.DistributedKnnEngine.try_new(base, base.shape[1], g, vc.GpuShardMode(mode),
                                           vc.DistanceMetric(metric))


def _assert_parity(metric, dg, ig, do, io, ctx=""):
    assert dg.shape == do.shape and ig.shape == io.shape, ctx
    assert np.array_equal(ig, io), (ctx, np.argwhere(ig != io)[:5])
    if metric == MINK:
        np.testing.assert_allclose(dg, do, rtol=1e-6, err_msg=ctx)
    else:
        assert np.array_equal(dg.view(np.uint32), do.view(np.uint32)), (
            ctx, np.argwhere(dg.view(np.uint32) != do.view(np.uint32))[:5])


def _data(vc, metric, n, q, d, seed):
    if metric in (HELL,):
        kind = vc.GEN_UNIFORM_SUM1
    elif metric in (L1, CHEB, JAC):
        kind = vc.GEN_UNIFORM
    elif metric == COS:
        kind = vc.GEN_NORMAL_UNIT
    else:
        kind = vc.GEN_NORMAL
    s = vc.config_seed(100 + seed)
    return (vc.gen_rows_host(kind, s, 0, 0, n, d), vc.gen_rows_host(kind, s, 1, 0, q, d))


@pytest.mark.parametrize("metric", range(10))
@pytest.mark.parametrize("d", [3, 17, 96, 128])
def test_parity_random(vc, orc, gpu, metric, d):
    base, qs = _data(vc, metric, 3000, 29, d, metric * 1000 + d)
    if metric == HAM:  # quantise so Hamming distances have many exact ties
        base, qs = np.round(base * 2) / 2, np.round(qs * 2) / 2
    eng = _engine(vc, base, metric)
    for k in (1, 10, 100):
        dg, ig = eng.search_arrays(qs, k)
        do, io = orc.knn_search(base, qs, k, metric)
        _assert_parity(metric, dg, ig, do, io, f"metric={metric} d={d} k={k}")


@pytest.mark.parametrize("metric", [L2, COS, L1, HELL])
def test_parity_many_queries_and_segments(vc, orc, gpu, metric):
    base, qs = _data(vc, metric, 20000, 300, 64, 7)
    eng = _engine(vc, base, metric)
    dg, ig = eng.search_arrays(qs, 50)
    do, io = orc.knn_search(base, qs, 50, metric)
    _assert_parity(metric, dg, ig, do, io)


def test_duplicates_and_ties(vc, orc, gpu):
    rng = np.random.default_rng(1)
    rows = rng.standard_normal((40, 8)).astype(np.float32)
    base = np.repeat(rows, 30, axis=0)  # 30 copies of each row: exact ties
    qs = rows[:5] + 0.01
    for metric in (L2, DOT, L1, CHEB):
        eng = _engine(vc, base, metric)
        dg, ig = eng.search_arrays(qs, 45)
        do, io = orc.knn_search(base, qs, 45, metric)
        _assert_parity(metric, dg, ig, do, io, f"metric={metric}")


def test_reference_kats(vc, gpu):
    Sm = vc.DistanceMetric
    # knn.rs:410-441
    data = np.array([[(i * i) * 0.1, i * 2.0, i + 5.0, i * 3.0] for i in range(50)], np.float32)
    eng = vc.CudaKnnEngine.new(data, 4, Sm.L2Squared)
    res = eng.search(data[10], 5)
    assert len(res) == 5 and res[0].id == 10 and abs(res[0].distance) < 1e-4
    # knn.rs:444-457
    eng = vc.CudaKnnEngine.new([0.0, 0.0, 1.0, 1.0, 2.0, 2.0], 2, Sm.L2Squared)
    r = eng.search_batch([0.1, 0.1, 1.9, 1.9], 1)
    assert len(r) == 2 and r[0][0].id == 0 and r[1][0].id == 2
    # knn.rs:460-474: empty queries and k = 0
    eng = vc.CudaKnnEngine.new([1.0, 2.0, 3.0, 4.0], 2, Sm.L2Squared)
    assert eng.search([], 5) == [] and eng.search_batch([], 5) == []
    assert eng.search([1.0, 2.0], 0) == []
    assert eng.search_batch([1.0, 2.0], 0) == [[]]
    # knn.rs:477-485: k > n
    eng = vc.CudaKnnEngine.new([0.0, 0.0, 1.0, 1.0, 2.0, 2.0], 2, Sm.L2Squared)
    assert len(eng.search([0.5, 0.5], 100)) == 3
    # knn.rs:488-503: cosine
    eng = vc.CudaKnnEngine.new([1.0, 0.0, 0.0, 1.0, -1.0, 0.0], 2, Sm.CosineSimilarity)
    r = eng.search([0.95, 0.05], 3)
    assert r[0].id == 0 and r[2].id == 2
    # knn.rs:506-521: dot
    eng = vc.CudaKnnEngine.new([1.0, 1.0, 2.0, 2.0, 3.0, 3.0], 2, Sm.DotProduct)
    r = eng.search([2.0, 3.0], 2)
    assert [x.id for x in r] == [2, 1] and r[0].distance == 15.0
    # knn.rs:524-532: getters
    eng = vc.CudaKnnEngine.new([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], 3, Sm.L2Squared)
    assert (eng.dimension(), eng.num_vectors(), eng.metric()) == (3, 2, Sm.L2Squared)
    # knn.rs:535-541: self queries
    data = [10.0, 20.0, 30.0, 40.0, 50.0, 60.0]
    eng = vc.CudaKnnEngine.new(data, 2, Sm.L2Squared)
    for i in range(3):
        r = eng.search(data[2 * i:2 * i + 2], 1)
        assert r[0].id == i and abs(r[0].distance) < 1e-4


def test_all_metrics_integration_dataset(vc, orc, gpu):
    # integration_tests.rs:121-161
    data = np.array([[0.8, 0.6], [0.8, 0.0], [0.0, 0.6], [0.1, 0.1], [-1.0, -1.0]], np.float32)
    q = np.array([[0.8, 0.6]], np.float32)
    for m in range(10):
        eng = _engine(vc, data, m)
        dg, ig = eng.search_arrays(q, 3)
        do, io = orc.knn_search(data, q, 3, m)
        _assert_parity(m, dg, ig, do, io, f"metric={m}")


def test_edge_shapes(vc, orc, gpu):
    rng = np.random.default_rng(5)
    for n, d, k in [(1, 1, 1), (1, 5, 10), (7, 1, 3), (64, 2, 64), (65, 3, 64), (300, 9, 300)]:
        base = rng.standard_normal((n, d)).astype(np.float32)
        qs = rng.standard_normal((4, d)).astype(np.float32)
        for m in (L2, COS, L1):
            eng = _engine(vc, base, m)
            dg, ig = eng.search_arrays(qs, k)
            do, io = orc.knn_search(base, qs, k, m)
            _assert_parity(m, dg, ig, do, io, f"n={n} d={d} k={k} m={m}")


def test_full_size_cosine_properties(vc, orc, gpu):
    """C2 shape (1M x 128, unit rows, k=100) on a query sample: sorted output,
    ids in range, and exact agreement with the oracle's full scan on the sample."""
    s = vc.config_seed(1)
    base = vc.gen_rows_host(vc.GEN_NORMAL_UNIT, s, 0, 0, 1_000_000, 128)
    qs = vc.gen_rows_host(vc.GEN_NORMAL_UNIT, s, 1, 0, 24, 128)
    eng = _engine(vc, base, COS)
    dg, ig = eng.search_arrays(qs, 100)
    assert (ig < 1_000_000).all()
    assert (np.diff(dg, axis=1) <= 0).all()
    do, io = orc.knn_search(base, qs, 100, COS)
    _assert_parity(COS, dg, ig, do, io)


@pytest.mark.parametrize("metric", [L1, CHEB, HELL])
def test_full_size_c4_sample(vc, orc, gpu, metric):
    """C4 shape (1M x 96 uniform rows, rows summing to 1 for Hellinger, k=10)
    on 150 queries (two 128-query tiles, the second partial): the CUDA-core
    scan's pivot-seeded candidates re-ranked exactly equal the oracle."""
    kind = vc.GEN_UNIFORM_SUM1 if metric == HELL else vc.GEN_UNIFORM
    s = vc.config_seed(3)
    base = vc.gen_rows_host(kind, s, 0, 0, 1_000_000, 96)
    qs = vc.gen_rows_host(kind, s, 1, 0, 150, 96)
    eng = _engine(vc, base, metric)
    dg, ig = eng.search_arrays(qs, 10)
    assert (ig < 1_000_000).all()
    assert (np.diff(dg, axis=1) >= 0).all()
    do, io = orc.knn_search(base, qs, 10, metric)
    _assert_parity(metric, dg, ig, do, io)


@pytest.mark.parametrize("d", [125, 126, 127])
def test_l2_fold_boundary(vc, orc, gpu, d):
    """Squared L2 folds -|x|^2/2 into two extra K columns while d + 2 <= 128;
    d = 127 keeps |x|^2 in the epilogue. Both sides of the boundary, with a
    wide value range."""
    base, qs = _data(vc, L2, 5000, 40, d, 900 + d)
    base[::7] *= 30.0
    eng = _engine(vc, base, L2)
    for k in (1, 64):
        dg, ig = eng.search_arrays(qs, k)
        do, io = orc.knn_search(base, qs, k, L2)
        _assert_parity(L2, dg, ig, do, io, f"d={d} k={k}")


def test_cosine_fp16_tiny_norms(vc, orc, gpu):
    """Cosine runs on fp16 unit rows; rows and queries with near-zero norms
    (where the reference's zero guard can fire) bypass the bound."""
    base, qs = _data(vc, COS, 4000, 30, 64, 77)
    base[5] *= 1e-6
    base[17] = 0.0
    qs[3] *= 1e-7
    qs[4] = 0.0
    eng = _engine(vc, base, COS)
    dg, ig = eng.search_arrays(qs, 20)
    do, io = orc.knn_search(base, qs, 20, COS)
    _assert_parity(COS, dg, ig, do, io)


def test_unproven_bound_fallback(vc, orc, gpu):
    """A single shard's starting bound comes from a low rank of the pivot
    minima (pivot rows: every 6th row at this size) and the select verifies
    it per query. Near rows placed only on pivot rows, fewer than k of them,
    make that bound cut true neighbours: the select must flag the queries and
    the exact fallback must return the oracle's answer."""
    n, d, k = 1_200_000, 32, 100
    rng = np.random.default_rng(11)
    qs = rng.standard_normal((3, d)).astype(np.float32)
    base = (rng.standard_normal((n, d)) * 3 + 20).astype(np.float32)
    for i in range(3):
        near = 6144 * (i * 60 + np.arange(60))  # pivot rows, 1024 pivot rows apart
        base[near] = qs[i] + 0.05 * rng.standard_normal((60, d)).astype(np.float32)
        mid = 6 * (20_000 + i * 300 + np.arange(200)) + 1  # rows outside the pivot set
        base[mid] = qs[i] + 0.5 * rng.standard_normal((200, d)).astype(np.float32)
    eng = _engine(vc, base, L2)
    vc.profile_reset()
    vc.profile_enable(True)
    dg, ig = eng.search_arrays(qs, k)
    vc.profile_enable(False)
    _, n_fb = vc.profile_read("knn_fallback")
    do, io = orc.knn_search(base, qs, k, L2)
    _assert_parity(L2, dg, ig, do, io)
    assert n_fb > 0
