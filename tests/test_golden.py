"""Golden fixtures (tests/golden/*.npz, written by tests/golden/make_golden.py).

CPU part: the host generator still produces the same inputs (checksums) and
the oracle still produces the committed outputs bit for bit, so a change to
either shows up here before any GPU comparison relies on them. GPU part:
libvrs's kNN and k-means against the committed outputs (kNN bit-exact; k-means
with the north star's bar: same iteration count, >= 99.9% equal assignments,
inertia within 1e-4 relative).
"""
import importlib.util
import os

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


def _mk():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MK = _mk()
KNN = np.load(os.path.join(HERE, "knn_golden.npz"))
KM = np.load(os.path.join(HERE, "kmeans_golden.npz"))


@pytest.fixture(scope="module")
def simd(orc):
    if not orc.has_avx512():
        pytest.skip("fixtures follow the AVX-512 path; this host has no AVX-512")
    return 1


@pytest.mark.parametrize("metric", range(10))
def test_oracle_knn_matches_fixture(vc, orc, simd, metric):
    base, qs = MK.knn_inputs(vc, metric)
    assert base.astype(np.float64).sum() == KNN[f"m{metric}_base_sum"]
    d, i = orc.knn_search(base, qs, MK.KNN_K, metric, use_simd=simd)
    assert np.array_equal(i, KNN[f"m{metric}_ids"])
    assert np.array_equal(d.view(np.uint32), KNN[f"m{metric}_dist_bits"])


def test_oracle_kmeans_matches_fixture(vc, orc, simd):
    x, init = MK.kmeans_inputs(vc)
    assert x.astype(np.float64).sum() == KM["x_sum"]
    for m in (L2, COS):
        c, a, it, inertia = orc.kmeans_fit(x, MK.KM_K, init, MK.KM_ITERS, 0.0, m, use_simd=simd)
        assert it == int(KM[f"m{m}_iters"])
        assert np.array_equal(a, KM[f"m{m}_assign"])
        assert np.array_equal(c.view(np.uint32), KM[f"m{m}_centroid_bits"])
        assert inertia == float(KM[f"m{m}_inertia"])


@pytest.mark.gpu
@pytest.mark.parametrize("metric", range(10))
def test_gpu_knn_matches_fixture(vc, gpu, metric):
    base, qs = MK.knn_inputs(vc, metric)
    eng = vc.DistributedKnnEngine.try_new(base, base.shape[1], 1, vc.GpuShardMode.Sharded,
                                          vc.DistanceMetric(metric))
    d, i = eng.search_arrays(qs, MK.KNN_K)
    eng.close()
    assert np.array_equal(i, KNN[f"m{metric}_ids"])
    if metric == MINK:  # cube root: CUDA cbrtf vs glibc cbrtf
        np.testing.assert_allclose(d, KNN[f"m{metric}_dist_bits"].view(np.float32), rtol=1e-6)
    else:
        assert np.array_equal(d.view(np.uint32), KNN[f"m{metric}_dist_bits"])


@pytest.mark.gpu
def test_gpu_knn_big_cosine_matches_fixture(vc, gpu):
    base, qs = MK.big_inputs(vc)
    eng = vc.CudaKnnEngine.new(base, base.shape[1], vc.DistanceMetric.CosineSimilarity)
    d, i = eng.search_arrays(qs, MK.BIG_K)
    eng.close()
    assert np.array_equal(i, KNN["big_ids"])
    assert np.array_equal(d.view(np.uint32), KNN["big_dist_bits"])


@pytest.mark.gpu
@pytest.mark.parametrize("metric", [L2, COS])
def test_gpu_kmeans_matches_fixture(vc, gpu, metric):
    x, init = MK.kmeans_inputs(vc)
    res = vc.CudaKMeansEngine.new().fit(x, MK.KM_D, MK.KM_K, MK.KM_ITERS, 0.0,
                                        vc.DistanceMetric(metric), init=init)
    assert res.iterations == int(KM[f"m{metric}_iters"])
    assert float((res.assignments == KM[f"m{metric}_assign"]).mean()) >= 0.999
    ref = float(KM[f"m{metric}_inertia"])
    assert abs(res.inertia - ref) <= 1e-4 * abs(ref)
