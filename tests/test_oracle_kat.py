"""CPU tests pinning the oracle to the reference's own known answers.

Known answers come from the reference's unit tests, read as text:
crates/vector-simd/src/scalar.rs:271-362 (metric values),
crates/vector-simd/src/avx512.rs:623-677 (SIMD vs scalar over dims 1..768),
crates/vector-cuda/src/knn.rs:410-542 (flat search KATs),
crates/vector-cuda/src/ddp/collective.rs:238-282 (top-k merge),
crates/vector-cuda/src/kmeans.rs:473-570 and
crates/vector-cuda/src/ddp/distributed_kmeans.rs:548-606 (k-means).
"""
import math

import numpy as np
import pytest

L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)
EPS = 1e-5


@pytest.mark.parametrize("simd", [0, 1])
def test_scalar_known_answers(orc, simd):
    # scalar.rs:271-362
    d = lambda m, a, b: orc.distance(m, a, b, simd)
    assert abs(d(DOT, [1, 2, 3], [4, 5, 6]) - 32.0) < EPS
    assert abs(d(L2, [1, 2, 3], [4, 6, 3]) - 25.0) < EPS
    assert abs(d(COS, [1, 2, 3], [1, 2, 3]) - 1.0) < EPS
    assert d(COS, [0, 0], [1, 2]) == 0.0
    assert abs(d(L1, [1, 5, 2], [4, 1, 6]) - 11.0) < EPS
    assert abs(d(L1, [1, 5, 2], [1, 5, 2])) < EPS
    assert abs(d(MINK, [1, 2, 3], [4, 2, 7]) - (27.0 + 64.0) ** (1 / 3)) < EPS
    assert abs(d(CHEB, [1, 10, 3], [5, 2, 4]) - 8.0) < EPS
    assert abs(d(HAM, [1, 2, 3, 4], [1, 9, 3, 8]) - 2.0) < EPS
    assert abs(d(MAHA, [0, 0], [3, 4]) - 5.0) < EPS
    assert abs(d(JAC, [1, 2, 0], [1, 0, 0]) - 2.0 / 3.0) < EPS
    assert abs(d(JAC, [1, 2, 0], [1, 2, 0])) < EPS
    assert abs(d(HELL, [0.25, 0.25], [0.25, 0.25])) < EPS


def _scalar_ref(m, a, b):
    """Textbook definitions of scalar.rs in float64 (tolerance reference)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    df = a - b
    if m == L2:
        return float((df * df).sum())
    if m == DOT:
        return float((a * b).sum())
    if m == L1:
        return float(np.abs(df).sum())
    if m == MINK:
        return float((np.abs(df) ** 3).sum() ** (1 / 3))
    if m == CHEB:
        return float(np.abs(df).max()) if len(a) else 0.0
    if m == HAM:
        return float((np.abs(df) > 1e-6).sum())
    if m == JAC:
        mn = np.minimum(np.abs(a), np.abs(b)).sum()
        mx = np.maximum(np.abs(a), np.abs(b)).sum()
        return 0.0 if mx <= 1e-9 else float(1 - mn / mx)
    if m == HELL:
        h = np.sqrt(np.abs(a)) - np.sqrt(np.abs(b))
        return float(math.sqrt(0.5 * (h * h).sum()))
    raise ValueError(m)


def test_simd_matches_scalar_semantics_and_emulation(orc):
    # avx512.rs:623-677: dims 1..768 with the formula vectors, rel < 1e-3.
    for dim in [1, 7, 8, 15, 16, 31, 32, 63, 64, 128, 768]:
        a = np.array([((i * 7 + 3) % 100) * 0.1 for i in range(dim)], np.float32)
        b = np.array([((i * 13 + 5) % 100) * 0.1 for i in range(dim)], np.float32)
        for m in (DOT, L2, L1, MINK, CHEB, HAM, JAC, HELL):
            v = orc.distance(m, a, b, 1)
            ref = _scalar_ref(m, a, b)
            assert abs(v - ref) / max(abs(ref), 1.0) < 1e-3, (dim, m, v, ref)
            # The portable emulation is bit-identical to the intrinsics.
            assert np.float32(v).tobytes() == np.float32(orc.distance(m, a, b, 0)).tobytes()


def test_emulation_bit_identical_random(orc):
    if not orc.has_avx512():
        pytest.skip("host has no AVX-512F")
    rng = np.random.default_rng(7)
    for dim in [1, 2, 3, 5, 16, 17, 31, 33, 64, 65, 96, 100, 128, 200, 768]:
        for _ in range(5):
            a = rng.standard_normal(dim).astype(np.float32)
            b = rng.standard_normal(dim).astype(np.float32)
            for m in range(10):
                x, y = orc.distance(m, a, b, 1), orc.distance(m, a, b, 0)
                assert np.float32(x).tobytes() == np.float32(y).tobytes(), (dim, m)


def _formula_dataset(n):
    # knn.rs:410-441 / distributed_knn.rs:270-310
    return np.array([[(i * i) * 0.1, i * 2.0, i + 5.0, i * 3.0] for i in range(n)], np.float32)


def _flat_ref(base, q, k, m):
    """Plain float64 brute force (independent check of the oracle's heap)."""
    sc = np.array([_scalar_ref(m, q, x) if m not in (COS, MAHA) else 0.0 for x in base])
    if m == MAHA:
        sc = np.sqrt(((base.astype(np.float64) - q) ** 2).sum(1))
    order = np.lexsort((np.arange(len(base)), -sc if m in (DOT, COS) else sc))
    return order[:k]


def test_knn_formula_dataset_matches_flat(orc):
    base = _formula_dataset(50)
    d, i = orc.knn_search(base, base[10:11], 5, L2)
    assert list(i[0]) == list(_flat_ref(base, base[10], 5, L2))
    assert i[0][0] == 10 and abs(d[0][0]) < 1e-4


def test_knn_reference_kats(orc):
    # knn.rs:444-541
    data = np.array([[0, 0], [1, 1], [2, 2]], np.float32)
    _, i = orc.knn_search(data, np.array([[0.1, 0.1], [1.9, 1.9]], np.float32), 1, L2)
    assert list(i[:, 0]) == [0, 2]
    d, i = orc.knn_search(data, np.array([[0.5, 0.5]], np.float32), 100, L2)
    assert i.shape == (1, 3)
    d, i = orc.knn_search(np.array([[1, 0], [0, 1], [-1, 0]], np.float32),
                          np.array([[0.95, 0.05]], np.float32), 3, COS)
    assert i[0][0] == 0 and i[0][2] == 2
    d, i = orc.knn_search(np.array([[1, 1], [2, 2], [3, 3]], np.float32),
                          np.array([[2, 3]], np.float32), 2, DOT)
    assert list(i[0]) == [2, 1] and list(d[0]) == [15.0, 10.0]
    data = np.array([[10, 20], [30, 40], [50, 60]], np.float32)
    for r in range(3):
        d, i = orc.knn_search(data, data[r:r + 1], 1, L2)
        assert i[0][0] == r and abs(d[0][0]) < 1e-4


def test_all_metrics_small(orc):
    # integration_tests.rs:121-161 dataset
    data = np.array([[0.8, 0.6], [0.8, 0.0], [0.0, 0.6], [0.1, 0.1], [-1.0, -1.0]], np.float32)
    q = np.array([[0.8, 0.6]], np.float32)
    for m in range(10):
        d, i = orc.knn_search(data, q, 3, m)
        assert i.shape == (1, 3)
        hib = m in (DOT, COS)
        dd = d[0] if not hib else -d[0]
        assert all(dd[j] <= dd[j + 1] for j in range(2)), m


def test_topk_reduce_kats(orc):
    # collective.rs:238-282
    d, i = orc.topk_reduce([([1.0, 5.0], [0, 1]), ([0.5, 4.0], [10, 11])], 2, L2)
    assert list(i) == [10, 0]
    d, i = orc.topk_reduce([([0.85, 0.40], [0, 1]), ([0.95, 0.70], [2, 3])], 3, COS)
    assert list(i) == [2, 0, 3]
    d, i = orc.topk_reduce([([2.0], [0]), ([1.0], [1])], 10, L2)
    assert list(i) == [1, 0]
    d, i = orc.topk_reduce([([1.0], [0])], 0, L2)
    assert len(i) == 0


def test_sharded_merge_equals_full_search(orc):
    # distributed_knn.rs:104-128 split + collective.rs merge == full search.
    rng = np.random.default_rng(3)
    base = rng.standard_normal((997, 17)).astype(np.float32)
    q = rng.standard_normal((9, 17)).astype(np.float32)
    for m in (L2, COS, L1):
        d_full, i_full = orc.knn_search(base, q, 7, m)
        g = 4
        chunk = -(-len(base) // g)
        parts = []
        for r in range(g):
            s, e = r * chunk, min(len(base), (r + 1) * chunk)
            dr, ir = orc.knn_search(base[s:e], q, 7, m)
            parts.append((dr, ir + s))
        for qi in range(len(q)):
            dm, im = orc.topk_reduce([(p[0][qi], p[1][qi]) for p in parts], 7, m)
            assert list(im) == list(i_full[qi])
            assert np.array_equal(dm, d_full[qi])


def test_kmeans_kats(orc):
    # distributed_kmeans.rs:596-606: single cluster -> mean.
    data = np.array([[1, 1], [3, 3], [5, 5], [7, 7]], np.float32)
    c, a, it, inertia = orc.kmeans_fit(data, 1, data[:1], 10, 1e-5, L2)
    assert np.allclose(c[0], [4, 4], atol=1e-3)
    # kmeans.rs:473-509: three separated clusters, inertia < 1.
    rows = [[0.1, -0.1, 0.05, -0.05]] * 50 + [[10.1, 9.9, 10.05, 9.95]] * 50 + \
           [[20.1, 19.9, 20.05, 19.95]] * 50
    data = np.array(rows, np.float32)
    init = data[[0, 50, 100]]
    c, a, it, inertia = orc.kmeans_fit(data, 3, init, 20, 1e-4, L2)
    assert inertia < 1.0 and it >= 1
    # k > n clamps (kmeans.rs:546-553).
    c, a, it, inertia = orc.kmeans_fit(np.array([[1, 2], [3, 4]], np.float32), 5,
                                       np.array([[1, 2], [3, 4]], np.float32), 10, 1e-4, L2)
    assert c.shape == (2, 2)
