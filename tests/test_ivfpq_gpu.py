"""IVF-PQ ADC search on the GPU (vrs_ivfpq_search) against the oracle's C
restatement of IvfPqIndex::search (orc_ivfpq_search, itself checked against
the Python restatement and the reference's PQ tests): ids, reported
distances bit for bit and result counts, on indexes with many exactly equal
ADC scores (few sub-centroids), empty lists, every probe count, k above the
number of candidates, and a C5b-sized quantiser."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


@pytest.fixture(scope="module")
def pq(orc):
    import ivfpq
    return ivfpq


def _index(rng, d, M, ksub, nlist, max_len, empty=(), nonneg=False):
    cb = rng.standard_normal(M * ksub * (d // M)).astype(np.float32)
    coarse = rng.standard_normal((nlist, d)).astype(np.float32)
    if nonneg:
        cb, coarse = np.abs(cb) * 0.1, np.abs(coarse)
    lists, nid = [], 0
    for c in range(nlist):
        n = 0 if c in empty else int(rng.integers(0, max_len))
        lists.append((np.arange(nid, nid + n, dtype=np.uint32) * 7 + 3,
                      rng.integers(0, ksub, (n, M)).astype(np.uint8)))
        nid += n
    return cb, coarse, lists


def _compare(vc, pq, cb, coarse, lists, M, ksub, metric, queries, cases):
    d = coarse.shape[1]
    idx = vc.IvfPqIndex(coarse, d, cb, M, ksub, lists, vc.DistanceMetric(metric))
    try:
        for k, nprobe in cases:
            gd, gi, gc = idx.search_batch(queries, k, nprobe)
            for qi, q in enumerate(queries):
                od, oi = pq.ivf_pq_search_c(q, k, nprobe, coarse, lists, cb, M, ksub, metric)
                n = len(oi)
                assert gc[qi] == n, (metric, k, nprobe, qi)
                assert np.array_equal(gi[qi, :n], oi), (metric, k, nprobe, qi)
                assert np.array_equal(gd[qi, :n].view(np.uint32), od.view(np.uint32)), (metric, k, nprobe, qi)
    finally:
        idx.close()


def test_hand_built_index(vc, gpu):
    # The worked example of the oracle tests (LUT [2, 0, 8, 0] for list 0).
    cb = np.array([0, 0, 1, 1, 0, 0, 2, 2], np.float32)
    coarse = np.array([[0, 0, 0, 0], [10, 10, 10, 10]], np.float32)
    lists = [(np.array([5, 6, 7]), np.array([[1, 1], [0, 0], [1, 0]], np.uint8)),
             (np.array([8]), np.array([[0, 0]], np.uint8))]
    idx = vc.IvfPqIndex(coarse, 4, cb, 2, 2, lists, vc.DistanceMetric.L2Squared)
    q = np.array([[1, 1, 2, 2]], np.float32)
    assert [(r.id, r.distance) for r in idx.search_with_nprobe(q, 2, 1)] == [(5, 0.0), (7, 8.0)]
    assert [(r.id, r.distance) for r in idx.search_with_nprobe(q, 4, 2)] == \
        [(5, 0.0), (7, 8.0), (6, 10.0), (8, 290.0)]
    assert idx.search_with_nprobe(q, 0, 2) == []
    assert [(r.id, r.distance) for r in idx.search_with_nprobe(q, 1, 0)] == [(5, 0.0)]  # nprobe clamped to 1
    idx.close()


@pytest.mark.parametrize("metric", [L2, DOT, COS, L1, CHEB, MAHA, HELL])
@pytest.mark.parametrize("ksub", [2, 16, 256])
def test_parity_random_indexes(vc, pq, gpu, metric, ksub):
    rng = np.random.default_rng(1000 * ksub + metric)
    d, M, nlist = 24, 6, 9  # M not a multiple of 4: the remainder codes
    cb, coarse, lists = _index(rng, d, M, ksub, nlist, 300, empty=(3,), nonneg=metric == HELL)
    qs = rng.standard_normal((40, d)).astype(np.float32)
    if metric == HELL:
        qs = np.abs(qs)
    _compare(vc, pq, cb, coarse, lists, M, ksub, metric, qs,
             [(1, 1), (10, 3), (100, 5), (2048, 0), (700, 20)])


def test_parity_tie_heavy_multiple_of_four(vc, pq, gpu):
    # One sub-centroid per sub-space in half the sub-spaces and two in the
    # rest: whole lists share a handful of ADC values.
    rng = np.random.default_rng(77)
    d, M, ksub, nlist = 32, 8, 2, 5
    cb, coarse, lists = _index(rng, d, M, ksub, nlist, 2000)
    for c in range(nlist):
        lists[c][1][:, ::2] = 0
    qs = rng.standard_normal((64, d)).astype(np.float32)
    _compare(vc, pq, cb, coarse, lists, M, ksub, L2, qs, [(1, 2), (50, 2), (333, 5), (2048, 5)])


def test_parity_c5b_quantiser_shape(vc, pq, gpu):
    # nlist 1024 over d = 96 with M = 16 sub-spaces of 256 sub-centroids and
    # 200k encoded rows, 200 queries at nprobe 32, k = 100.
    rng = np.random.default_rng(5)
    d, M, ksub, nlist = 96, 16, 256, 1024
    cb, coarse, lists = _index(rng, d, M, ksub, nlist, 400)
    qs = (coarse[rng.integers(0, nlist, 200)] + 0.3 * rng.standard_normal((200, d))).astype(np.float32)
    _compare(vc, pq, cb, coarse, lists, M, ksub, L2, qs, [(100, 32)])


def test_empty_index_and_k_zero(vc, gpu):
    rng = np.random.default_rng(1)
    cb = rng.standard_normal(4 * 4 * 2).astype(np.float32)
    coarse = rng.standard_normal((3, 8)).astype(np.float32)
    lists = [(np.zeros(0, np.uint32), np.zeros((0, 4), np.uint8))] * 3
    idx = vc.IvfPqIndex(coarse, 8, cb, 4, 4, lists, vc.DistanceMetric.L2Squared)
    _, _, c = idx.search_batch(rng.standard_normal((5, 8)).astype(np.float32), 10, 2)
    assert list(c) == [0] * 5
    idx.close()
