"""CPU checks of the IVF-PQ ADC oracle (oracle/ivfpq.py), no GPU.

Pinned on the reference's own PQ tests (crates/vector-index/src/ivf/pq.rs:
test_pq_adc_lut, test_pq_compute_distance_with_lut_remainder_unroll), on the
f32 summation order of compute_distance_with_lut (pq.rs:270-296), on the
tie behaviour that follows from std's BinaryHeap algorithm, and on a
hand-built two-list index whose ADC distances are worked out by hand.
"""
import numpy as np
import pytest

L2, DOT, COS = 0, 1, 2


@pytest.fixture(scope="module")
def pq(orc):
    import ivfpq
    return ivfpq


def test_kat_adc_lut(pq):
    # pq.rs test_pq_adc_lut
    cb = [0, 0, 1, 1, 0, 0, 2, 2]
    lut = pq.pq_adc_lut([1, 1, 2, 2], cb, 2, 2, L2)
    assert list(lut) == [2.0, 0.0, 8.0, 0.0]
    assert pq.pq_distance_with_lut([1, 1], lut, 2) == 0.0
    assert pq.pq_distance_with_lut([0, 0], lut, 2) == 10.0


def test_kat_remainder_unroll(pq):
    # pq.rs test_pq_compute_distance_with_lut_remainder_unroll: M = 5
    cb = [0.0, 1.0] * 5
    lut = pq.pq_adc_lut([1.0] * 5, cb, 5, 2, L2)
    assert abs(pq.pq_distance_with_lut([1] * 5, lut, 2)) < 1e-5
    assert abs(pq.pq_distance_with_lut([0] * 5, lut, 2) - 5.0) < 1e-5


def test_pairwise_summation_order(pq):
    # (d0 + d1) + (d2 + d3) in f32: 1e8 absorbs each 1, so the pairs cancel to
    # 0 where a running sum would end at 1.
    lut = np.array([1e8, 0, 1, 0, -1e8, 0, 1, 0], np.float32)
    assert pq.pq_distance_with_lut([0, 0, 0, 0], lut, 2) == 0.0
    s = np.float32(0)
    for v in (1e8, 1, -1e8, 1):
        s = np.float32(s + np.float32(v))
    assert s == 1.0


def test_rust_heap_tie_order(pq):
    # Equal keys: push a, b, c then pop returns a, b, c (traced through
    # sift_up / sift_down_to_bottom); the search reverses the pops, so its
    # output lists equal scores latest-inserted first.
    h = pq.RustMaxHeap()
    for name in "abc":
        h.push((1.0, name))
    assert [h.pop()[1] for _ in range(3)] == ["a", "b", "c"]
    rng = np.random.default_rng(3)
    vals = rng.standard_normal(200).astype(np.float32)
    h = pq.RustMaxHeap()
    for i, v in enumerate(vals):
        h.push((v, i))
    popped = [h.pop()[0] for _ in range(len(vals))]
    assert popped == sorted(vals, reverse=True)


def _hand_index():
    cb = np.array([0, 0, 1, 1, 0, 0, 2, 2], np.float32)          # M = 2, ksub = 2, dsub = 2
    coarse = np.array([[0, 0, 0, 0], [10, 10, 10, 10]], np.float32)
    lists = [(np.array([5, 6, 7]), np.array([[1, 1], [0, 0], [1, 0]], np.uint8)),
             (np.array([8]), np.array([[0, 0]], np.uint8))]
    return cb, coarse, lists


def test_hand_built_index(pq):
    cb, coarse, lists = _hand_index()
    q = [1, 1, 2, 2]
    # nprobe 1: list 0 only, LUT [2, 0, 8, 0]: id 5 -> 0, id 6 -> 10, id 7 -> 8
    assert pq.ivf_pq_search(q, 2, 1, coarse, lists, cb, 2, 2, L2) == [(5, 0.0), (7, 8.0)]
    # nprobe 2: residual q - 10 = [-9,-9,-8,-8]: LUT [162, 200, 128, 200], id 8 -> 290
    assert pq.ivf_pq_search(q, 4, 2, coarse, lists, cb, 2, 2, L2) == \
        [(5, 0.0), (7, 8.0), (6, 10.0), (8, 290.0)]
    # k = 0 and nprobe 0 (clamped to 1, mod.rs:275)
    assert pq.ivf_pq_search(q, 0, 2, coarse, lists, cb, 2, 2, L2) == []
    assert pq.ivf_pq_search(q, 1, 0, coarse, lists, cb, 2, 2, L2) == [(5, 0.0)]
    # no coarse centroids: empty result
    assert pq.ivf_pq_search(q, 3, 2, np.zeros((0, 4), np.float32), [], cb, 2, 2, L2) == []


@pytest.mark.parametrize("metric", [L2, DOT, COS])
def test_search_matches_sorted_scan_without_ties(pq, orc, metric):
    # Random codebooks and codes: every ADC distance distinct, so the heap's
    # result is the k best of the probed lists by score.
    rng = np.random.default_rng(10 + metric)
    d, M, ksub, nlist, k, nprobe = 8, 4, 16, 6, 10, 3
    cb = rng.standard_normal(M * ksub * (d // M)).astype(np.float32)
    coarse = rng.standard_normal((nlist, d)).astype(np.float32)
    lists, nid = [], 0
    for c in range(nlist):
        n = int(rng.integers(0, 30))
        lists.append((np.arange(nid, nid + n), rng.integers(0, ksub, (n, M)).astype(np.uint8)))
        nid += n
    q = rng.standard_normal(d).astype(np.float32)
    got = pq.ivf_pq_search(q, k, nprobe, coarse, lists, cb, M, ksub, metric)
    cand = []
    for cid, _ in orc.find_top_centroids(q, coarse, nprobe, metric):
        ids, codes = lists[cid]
        lut = pq.pq_adc_lut((q - coarse[cid]).astype(np.float32), cb, M, ksub, metric)
        cand += [(int(i), pq.pq_distance_with_lut(cd, lut, ksub)) for i, cd in zip(ids, codes)]
    assert len({v for _, v in cand}) == len(cand)
    cand.sort(key=lambda t: t[1], reverse=metric in (DOT, COS))
    assert got == cand[:k]


def test_encode(pq):
    # pq.rs:178-201 with the codebooks of test_pq_adc_lut: exact sub-centroids
    # encode to themselves; otherwise the nearest per sub-space, lower index
    # on equal distances (kmeans.rs:297-305).
    cb = [0, 0, 1, 1, 0, 0, 2, 2]
    assert list(pq.pq_encode([1, 1, 2, 2], cb, 2, 2, L2)) == [1, 1]
    assert list(pq.pq_encode([0.1, 0.0, 0.4, 0.5], cb, 2, 2, L2)) == [0, 0]
    assert list(pq.pq_encode([0.5, 0.5, 1.0, 1.0], cb, 2, 2, L2)) == [0, 0]  # ties -> 0


@pytest.mark.parametrize("metric", [L2, DOT, COS, 3])
@pytest.mark.parametrize("ksub", [2, 16])
def test_c_search_matches_python(pq, orc, metric, ksub):
    # The C form (for large parity cases) against the Python restatement, on
    # indexes with many exact ADC ties (ksub = 2: few distinct codes) and
    # without, for several k and nprobe.
    rng = np.random.default_rng(100 * ksub + metric)
    d, M, nlist = 12, 6, 7
    cb = rng.standard_normal(M * ksub * (d // M)).astype(np.float32)
    coarse = rng.standard_normal((nlist, d)).astype(np.float32)
    lists, nid = [], 0
    for c in range(nlist):
        n = int(rng.integers(0, 40)) if c != 2 else 0  # list 2 stays empty
        lists.append((np.arange(nid, nid + n), rng.integers(0, ksub, (n, M)).astype(np.uint8)))
        nid += n
    for t in range(4):
        q = rng.standard_normal(d).astype(np.float32)
        for k, nprobe in ((1, 1), (7, 3), (25, 7), (500, 0)):
            py = pq.ivf_pq_search(q, k, nprobe, coarse, lists, cb, M, ksub, metric)
            dc, ic = pq.ivf_pq_search_c(q, k, nprobe, coarse, lists, cb, M, ksub, metric)
            assert [(int(i), np.float32(v)) for i, v in zip(ic, dc)] == \
                [(i, np.float32(v)) for i, v in py], (metric, ksub, k, nprobe, t)
