"""GPU parity of Lloyd k-means against the CPU oracle, through the C ABI.

The bar (north star): identical init and iteration count, >= 99.9% equal
assignments, inertia within 1e-4 relative. The GPU assignment uses the
reference's exact pair arithmetic; centroid sums are exact fixed-point
integers, so in practice assignments agree exactly. Reference tests
mirrored: crates/vector-cuda/src/kmeans.rs:469-577,
crates/vector-cuda/src/ddp/distributed_kmeans.rs:544-642.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


def _mixture(vc, n, d, K, sigma, seed):
    s = vc.config_seed(200 + seed)
    c = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, K, d)
    return vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, n, d, c, K, sigma)


def _check(res, c_o, a_o, it_o, in_o):
    assert res.iterations == it_o
    agree = float((res.assignments == a_o).mean())
    assert agree >= 0.999, agree
    assert abs(res.inertia - in_o) <= 1e-4 * max(abs(in_o), 1e-30), (res.inertia, in_o)
    return agree


@pytest.mark.parametrize("metric", [L2, COS, DOT, L1, HELL, CHEB])
def test_parity_mixture(vc, orc, gpu, metric):
    x = _mixture(vc, 20000, 32, 64, 0.1, metric)
    if metric == HELL:
        x = np.abs(x)
    K = 64
    init = x[:K]
    eng = vc.CudaKMeansEngine.new()
    res = eng.fit(x, 32, K, 8, 0.0, vc.DistanceMetric(metric), init=init)
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, K, init, 8, 0.0, metric)
    agree = _check(res, c_o, a_o, it_o, in_o)
    if metric == L2:
        assert agree == 1.0
        np.testing.assert_allclose(res.centroids, c_o, rtol=1e-6, atol=1e-6)


def test_parity_c3_shape_small(vc, orc, gpu):
    """C3 distribution (1024 centres N(0,1), sigma 0.1, D=128, init = first
    K points, tol = 0) at 100k points."""
    x = _mixture(vc, 100_000, 128, 1024, 0.1, 3)
    init = x[:1024]
    res = vc.CudaKMeansEngine.new().fit(x, 128, 1024, 5, 0.0, vc.DistanceMetric.L2Squared,
                                        init=init)
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, 1024, init, 5, 0.0, L2)
    _check(res, c_o, a_o, it_o, in_o)


def test_reference_kats(vc, gpu):
    M = vc.DistanceMetric
    eng = vc.CudaKMeansEngine.new()
    rows = [[0.1, -0.1, 0.05, -0.05]] * 50 + [[10.1, 9.9, 10.05, 9.95]] * 50 + \
           [[20.1, 19.9, 20.05, 19.95]] * 50
    data = np.array(rows, np.float32)
    r = eng.fit(data, 4, 3, 20, 1e-4, M.L2Squared, init=data[[0, 50, 100]])
    assert r.k == 3 and r.dimension == 4 and r.iterations > 0 and r.inertia < 1.0
    r = eng.fit([1.0, 1.0, 1.1, 0.9, 0.9, 1.1], 2, 1, 10, 1e-4, M.L2Squared)
    assert r.k == 1 and abs(r.centroid(0)[0] - 1.0) < 0.1 and abs(r.centroid(0)[1] - 1.0) < 0.1
    assert eng.fit([], 4, 3, 10, 1e-4, M.L2Squared).k == 0
    assert eng.fit([1.0, 2.0], 2, 0, 10, 1e-4, M.L2Squared).k == 0
    assert eng.fit([1.0, 2.0, 3.0, 4.0], 2, 5, 10, 1e-4, M.L2Squared).k == 2
    d = [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0, 0.9, 0.1, 0.0]
    assert eng.fit(d, 3, 3, 10, 1e-4, M.CosineSimilarity).k == 3
    assert eng.fit(d, 3, 3, 10, 1e-4, M.DotProduct).k == 3
    hd = (np.arange(20 * 128, dtype=np.float32) * 0.01)
    r = eng.fit(hd, 128, 4, 5, 1e-3, M.L2Squared)
    assert r.k == 4 and r.dimension == 128
    # distributed_kmeans.rs:596-606: single cluster centroid = mean
    r = eng.fit([1.0, 1.0, 3.0, 3.0, 5.0, 5.0, 7.0, 7.0], 2, 1, 10, 1e-5, M.L2Squared)
    assert np.allclose(r.centroid(0), [4.0, 4.0], atol=1e-3)


def test_tolerance_stop_and_determinism(vc, orc, gpu):
    x = _mixture(vc, 5000, 16, 8, 0.05, 9)
    init = x[:8]
    eng = vc.CudaKMeansEngine.new()
    r1 = eng.fit(x, 16, 8, 50, 1e-6, vc.DistanceMetric.L2Squared, init=init)
    r2 = eng.fit(x, 16, 8, 50, 1e-6, vc.DistanceMetric.L2Squared, init=init)
    assert r1.iterations < 50
    assert np.array_equal(r1.centroids.view(np.uint32), r2.centroids.view(np.uint32))
    assert r1.inertia == r2.inertia
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, 8, init, 50, 1e-6, 0)
    _check(r1, c_o, a_o, it_o, in_o)


@pytest.mark.parametrize("scale", [1e4, 1e-4, 1e-12])
@pytest.mark.parametrize("metric", [L2, DOT])
def test_operand_scale_extremes(vc, orc, gpu, metric, scale):
    """The tensor-core assignment scales points and centroids by one power of
    two into fp16's range: data far from unit magnitude (and initial
    centroids larger than the data) must give the oracle's result."""
    x = (_mixture(vc, 20000, 24, 32, 0.1, 11) * scale).astype(np.float32)
    K = 32
    init = x[:K].copy()
    init[0] *= 4.0  # an initial centroid outside the data's range
    res = vc.CudaKMeansEngine.new().fit(x, 24, K, 5, 0.0, vc.DistanceMetric(metric), init=init)
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, K, init, 5, 0.0, metric)
    _check(res, c_o, a_o, it_o, in_o)


@pytest.mark.parametrize("metric", [L2, COS, DOT])
def test_duplicate_centroids_exact_ties(vc, orc, gpu, metric):
    """Initial centroids with exact duplicates: every point near a duplicated
    pair has two candidates with equal exact scores inside its bound, so the
    multi-candidate exact pass must pick the lower index (kmeans.rs:361-407,
    strict comparison); points with a single in-bound candidate are assigned
    without being re-scored, and the inertia still comes from exact
    distances."""
    x = _mixture(vc, 30000, 48, 96, 0.1, 40 + metric)
    K = 96
    init = np.array(x[:K])
    init[1::2] = init[0::2]  # pairs (0,1), (2,3), ... coincide
    res = vc.CudaKMeansEngine.new().fit(x, 48, K, 6, 0.0, vc.DistanceMetric(metric), init=init)
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, K, init, 6, 0.0, metric)
    agree = _check(res, c_o, a_o, it_o, in_o)
    if metric == L2:
        assert agree == 1.0
        assert abs(res.inertia - in_o) <= 1e-6 * abs(in_o)
