"""CPU checks of the IVF coarse-quantiser oracle (no GPU).

Pins `oracle.find_nearest_centroid` / `find_top_centroids` (literal
restatements of crates/vector-index/src/ivf/kmeans.rs:264-356) on the
reference's own known-answer tests (kmeans.rs:420-441, 477-525;
crates/vector-mpi/src/distributed_kmeans.rs:504-527), and the batched form
the GPU tests compare against to the literal loops, ties included.
"""
import numpy as np
import pytest

L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


def test_kat_find_top_centroids_l2(orc):
    # kmeans.rs:420-441
    c = np.array([[0, 0], [5, 5], [10, 10]], np.float32)
    top2 = orc.find_top_centroids([1.0, 1.0], c, 2, L2)
    assert [i for i, _ in top2] == [0, 1]


def test_kat_find_top_centroids_cosine_edges(orc):
    # kmeans.rs:477-525: highest similarity first, nprobe 0, nprobe > K
    c = np.array([[1, 0], [0, 1], [-1, 0]], np.float32)
    q = [0.99, 0.01]
    top = orc.find_top_centroids(q, c, 2, COS)
    assert len(top) == 2 and top[0][0] == 0
    assert orc.find_top_centroids(q, c, 0, COS) == []
    assert len(orc.find_top_centroids(q, c, 100, COS)) == 3


def test_kat_find_nearest_centroid(orc):
    # distributed_kmeans.rs:504-527 (same contract as kmeans.rs:264-309)
    idx, dist = orc.find_nearest_centroid([1.0, 1.0], np.array([[0, 0], [10, 10]], np.float32), L2)
    assert idx == 0 and abs(dist - 2.0) < 1e-5
    idx, _ = orc.find_nearest_centroid([1.0, 0.0], np.array([[1, 0], [0, 1]], np.float32), DOT)
    assert idx == 0


def test_find_nearest_centroid_empty(orc):
    # kmeans.rs:272-277: no centroids -> the loop's initial values
    assert orc.find_nearest_centroid([1.0], np.zeros((0, 1), np.float32), L2) == (0, np.inf)
    assert orc.find_nearest_centroid([1.0], np.zeros((0, 1), np.float32), COS) == (0, -np.inf)


def _centroids(metric, K, d, seed):
    rng = np.random.default_rng(seed)
    c = rng.random((K, d), dtype=np.float32) if metric in (L1, CHEB, JAC, HELL, HAM) else \
        rng.standard_normal((K, d), dtype=np.float32)
    if metric == HAM:
        c = np.round(c * 3).astype(np.float32)
    if metric == HELL:
        c /= c.sum(1, keepdims=True)
    c[1::7] = c[0::7][: len(c[1::7])]  # exact duplicates: equal scores, index order decides
    return c


@pytest.mark.parametrize("metric", range(10))
def test_batch_matches_literal(orc, metric):
    K, d, nq = 40, 19, 12
    c = _centroids(metric, K, d, 10 + metric)
    q = _centroids(metric, nq, d, 90 + metric)
    for nprobe in (1, 5, K, K + 3):
        sb, ib = orc.find_top_centroids_batch(q, c, nprobe, metric, nthreads=2)
        for r in range(nq):
            lit = orc.find_top_centroids(q[r], c, nprobe, metric)
            assert [i for i, _ in lit] == list(ib[r]), (metric, nprobe, r)
            assert np.array_equal(np.array([v for _, v in lit], np.float32).view(np.uint32),
                                  sb[r].view(np.uint32))
    for r in range(nq):
        idx, v = orc.find_nearest_centroid(q[r], c, metric)
        sb, ib = orc.find_top_centroids_batch(q[r:r + 1], c, 1, metric, nthreads=1)
        assert idx == ib[0, 0] and np.float32(v).view(np.uint32) == sb[0, 0].view(np.uint32)


def test_rooted_tie_orders_by_index(orc):
    # Two distinct squared sums (6.25 and 6.25 + 2^-21) whose square roots
    # round to the same 2.5: the reference sorts the reported values stably,
    # so index order decides, while ordering by the sum would not.
    q = np.zeros(4, np.float32)
    a = np.array([2.5, 0, 0, 0], np.float32)
    b = np.array([2.5, 0.75 * 2 ** -10, 0, 0], np.float32)
    assert orc.rank_key(MAHA, q, a) < orc.rank_key(MAHA, q, b)
    assert orc.distance(MAHA, q, a) == orc.distance(MAHA, q, b)
    c = np.stack([b, a] * 10)
    assert [i for i, _ in orc.find_top_centroids(q, c, 3, MAHA)] == [0, 1, 2]
    _, ib = orc.find_top_centroids_batch(q[None], c, 3, MAHA)
    assert list(ib[0]) == [0, 1, 2]
    assert orc.find_nearest_centroid(q, c, MAHA)[0] == 0
