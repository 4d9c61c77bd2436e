"""GPU parity of IVF coarse probing and assignment, through the C ABI.

`vrs_ivf_find_top_centroids` and `vrs_ivf_assign` answer the reference's
KMeans::find_top_centroids / find_nearest_centroid
(crates/vector-index/src/ivf/kmeans.rs:264-356) for batches on the GPU. The
bar: centroid indices identical to the oracle's (reported value, index)
order and values bit-identical; Minkowski values within 1e-6 relative
(CUDA's cbrtf against glibc's), its indices compared as sets inside runs of
values that close. Cases: the reference's own tests (kmeans.rs:420-441,
477-525; crates/vector-mpi/src/distributed_kmeans.rs:504-527), every metric
with duplicated centroids, nprobe at 1, inside, at and beyond K, an IVF-sized
quantiser (K = 4096, d = 128) and distinct sums whose roots round equal.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


def _rows(vc, metric, n, d, seed, stream):
    if metric == HELL:
        kind = vc.GEN_UNIFORM_SUM1
    elif metric in (L1, CHEB, JAC, HAM):
        kind = vc.GEN_UNIFORM
    elif metric == COS:
        kind = vc.GEN_NORMAL_UNIT
    else:
        kind = vc.GEN_NORMAL
    x = vc.gen_rows_host(kind, vc.config_seed(300 + seed), stream, 0, n, d)
    if metric == HAM:  # few distinct values: many exact Hamming ties
        x = np.round(x * 3).astype(np.float32)
    return x


def _assert_probe(metric, sg, ig, so, io, ctx=""):
    assert sg.shape == so.shape and ig.shape == io.shape, ctx
    if metric != MINK:
        assert np.array_equal(ig, io), (ctx, np.argwhere(ig != io)[:5])
        assert np.array_equal(sg.view(np.uint32), so.view(np.uint32)), (
            ctx, np.argwhere(sg.view(np.uint32) != so.view(np.uint32))[:5])
        return
    np.testing.assert_allclose(sg, so, rtol=1e-6, err_msg=ctx)
    for r in range(so.shape[0]):
        v = so[r].astype(np.float64)
        j = 0
        while j < len(v):  # runs of values within 2e-6 relative of each other
            e = j + 1
            while e < len(v) and abs(v[e] - v[e - 1]) <= 2e-6 * abs(v[e]):
                e += 1
            if e - j == 1:
                assert ig[r, j] == io[r, j], (ctx, r, j)
            elif e < len(v):
                assert set(ig[r, j:e]) == set(io[r, j:e]), (ctx, r, j)
            j = e


def test_reference_kats(vc, gpu):
    Sm = vc.DistanceMetric
    # kmeans.rs:420-441
    top2 = vc.KMeans.find_top_centroids([1.0, 1.0], [0, 0, 5, 5, 10, 10], 2, 2, Sm.L2Squared)
    assert [i for i, _ in top2] == [0, 1] and top2[0][1] == 2.0
    # kmeans.rs:477-525: highest similarity first, nprobe 0, nprobe > K
    c = [1.0, 0.0, 0.0, 1.0, -1.0, 0.0]
    top = vc.KMeans.find_top_centroids([0.99, 0.01], c, 2, 2, Sm.CosineSimilarity)
    assert len(top) == 2 and top[0][0] == 0
    assert vc.KMeans.find_top_centroids([0.99, 0.01], c, 2, 0, Sm.CosineSimilarity) == []
    assert len(vc.KMeans.find_top_centroids([0.99, 0.01], c, 2, 100, Sm.CosineSimilarity)) == 3
    # distributed_kmeans.rs:504-527
    idx, dist = vc.KMeans.find_nearest_centroid([1.0, 1.0], [0, 0, 10, 10], 2, Sm.L2Squared)
    assert idx == 0 and abs(dist - 2.0) < 1e-5
    idx, _ = vc.KMeans.find_nearest_centroid([1.0, 0.0], [1, 0, 0, 1], 2, Sm.DotProduct)
    assert idx == 0


def test_no_centroids(vc, gpu):
    # kmeans.rs:272-277: no centroids -> index 0 and the loop's initial value
    for metric, init in ((L2, np.inf), (COS, -np.inf)):
        cq = vc.CoarseQuantizer(np.zeros((0, 3), np.float32), 3, vc.DistanceMetric(metric))
        ix, sc = cq.assign(np.ones((4, 3), np.float32))
        assert list(ix) == [0] * 4 and np.all(sc == init)
        s, i = cq.find_top_centroids(np.ones((2, 3), np.float32), 8)
        assert s.shape == (2, 0) and i.shape == (2, 0)
        cq.close()


@pytest.mark.parametrize("metric", range(10))
def test_probe_parity(vc, orc, gpu, metric):
    K, d, nq = 300, 40, 257
    c = _rows(vc, metric, K, d, metric, 0)
    c[1::9] = c[0::9][: len(c[1::9])]  # duplicated centroids: exact ties, index order
    q = _rows(vc, metric, nq, d, metric, 1)
    cq = vc.CoarseQuantizer(c, d, vc.DistanceMetric(metric))
    for nprobe in (1, 16, K, K + 10):
        sg, ig = cq.find_top_centroids(q, nprobe)
        so, io = orc.find_top_centroids_batch(q, c, nprobe, metric)
        _assert_probe(metric, sg, ig, so, io, f"metric={metric} nprobe={nprobe}")
    ixg, scg = cq.assign(q)
    so, io = orc.find_top_centroids_batch(q, c, 1, metric)
    _assert_probe(metric, scg[:, None], ixg[:, None], so, io, f"assign metric={metric}")
    for r in (0, 17, nq - 1):  # the literal loop of kmeans.rs:264-309
        idx, v = orc.find_nearest_centroid(q[r], c, metric)
        assert ixg[r] == idx and (metric == MINK or scg[r] == v)
    cq.close()


@pytest.mark.parametrize("metric", [L2, COS, DOT, HELL])
def test_probe_ivf_sized(vc, orc, gpu, metric):
    # An IVF quantiser of nlist = 4096 over d = 128 (the tensor-core scan for
    # L2/cosine/dot), probed at nprobe = 32 and used to assign base rows.
    K, d, nq = 4096, 128, 600
    c = _rows(vc, metric, K, d, 20 + metric, 0)
    q = _rows(vc, metric, nq, d, 20 + metric, 1)
    cq = vc.CoarseQuantizer(c, d, vc.DistanceMetric(metric))
    sg, ig = cq.find_top_centroids(q, 32)
    so, io = orc.find_top_centroids_batch(q, c, 32, metric)
    _assert_probe(metric, sg, ig, so, io, f"metric={metric}")
    ixg, scg = cq.assign(q)
    assert np.array_equal(ixg, io[:, 0]) and np.array_equal(scg.view(np.uint32), so[:, 0].view(np.uint32))
    cq.close()


def test_rooted_tie_orders_by_index(vc, gpu):
    # Squared sums 6.25 and 6.25 + 2^-21 both have the root 2.5 in f32: the
    # reference's stable sort keeps index order (0, 1, 2, ...), where the kNN
    # ranking by the sum alone would put the odd rows first. With 20 equal
    # values the probe must also widen its fetch past the boundary run.
    a = np.array([2.5, 0, 0, 0], np.float32)
    b = np.array([2.5, 0.75 * 2 ** -10, 0, 0], np.float32)
    c = np.stack([b, a] * 10)
    cq = vc.CoarseQuantizer(c, 4, vc.DistanceMetric(MAHA))
    q = np.zeros((2, 4), np.float32)
    for nprobe in (1, 3, 12, 20):
        s, i = cq.find_top_centroids(q, nprobe)
        assert i.tolist() == [list(range(nprobe))] * 2 and np.all(s == 2.5)
    ix, sc = cq.assign(q)
    assert list(ix) == [0, 0] and np.all(sc == 2.5)
    cq.close()


@pytest.mark.parametrize("metric", [L2, COS])
def test_train_save_load_probe_loop(vc, orc, gpu, tmp_path, metric):
    # The training -> index loop: k-means on the GPU, the centroids written as
    # the reference's standalone centroid file (ivf/serializer.rs:255-307),
    # read back (:309-370) into a coarse quantiser, which then assigns the
    # training rows and probes queries exactly as the oracle's literal loops
    # over the loaded centroids do.
    s = vc.config_seed(600 + metric)
    n, d, K = 12_000, 32, 64
    centres = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, K, d)
    x = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, n, d, centres, K, 0.05)
    M = vc.DistanceMetric(metric)
    res = vc.CudaKMeansEngine.new().fit(x, d, K, 25, 0.0, M)
    p = tmp_path / "coarse.centroids"
    vc.IvfPqSerializer.save_centroid_file(p, res.centroids, d, res.k, M, res.iterations,
                                          res.inertia)
    ld = vc.IvfPqSerializer.load_centroid_file(p)
    assert (ld.k, ld.dimension, ld.metric, ld.iterations) == (res.k, d, M, res.iterations)
    assert np.array_equal(ld.centroids.view(np.uint32), res.centroids.view(np.uint32))
    assert ld.inertia == np.float32(res.inertia)
    cq = vc.CoarseQuantizer(ld.centroids, d, ld.metric)
    ix, sc = cq.assign(x)
    so, io = orc.find_top_centroids_batch(x, ld.centroids, 1, metric)
    assert np.array_equal(ix, io[:, 0]) and np.array_equal(sc.view(np.uint32), so[:, 0].view(np.uint32))
    # The last Lloyd assignment was made against the centroids before the
    # final update; on this separated mixture the two agree nearly everywhere.
    assert float((ix == res.assignments).mean()) >= 0.95
    q = vc.gen_rows_host(vc.GEN_MIXTURE, s, 1, 0, 300, d, centres, K, 0.05)
    sg, ig = cq.find_top_centroids(q, 8)
    so, io = orc.find_top_centroids_batch(q, ld.centroids, 8, metric)
    _assert_probe(metric, sg, ig, so, io, "loop")
    for r in (0, 299):
        lit = orc.find_top_centroids(q[r], ld.centroids, 8, metric)
        assert [i for i, _ in lit] == list(ig[r])
    cq.close()


def test_nprobe_at_the_search_limit(vc, orc, gpu):
    # One search returns at most 2048 neighbours. Plain metrics probe 2048 of
    # 3000 centroids directly; the rooted metrics need the entry after the
    # boundary, so 2048 < K is refused with InvalidConfig and 2047 works.
    K, d, nq = 3000, 16, 5
    c = _rows(vc, L2, K, d, 77, 0)
    q = _rows(vc, L2, nq, d, 77, 1)
    for metric, p in ((L2, 2048), (MAHA, 2047)):
        cq = vc.CoarseQuantizer(c, d, vc.DistanceMetric(metric))
        sg, ig = cq.find_top_centroids(q, p)
        so, io = orc.find_top_centroids_batch(q, c, p, metric)
        _assert_probe(metric, sg, ig, so, io, f"metric={metric} nprobe={p}")
        if metric == MAHA:
            with pytest.raises(vc.CudaError) as e:
                cq.find_top_centroids(q, 2048)
            assert e.value.status == 5
        cq.close()
