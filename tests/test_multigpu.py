"""Multi-GPU parity through the C ABI (needs 2 or more GPUs; skipped otherwise).

* one process, several GPUs (vrs_knn_create / vrs_kmeans_fit with
  num_gpus > 1): GpuShardMode::Sharded row shards merged on the GPU after an
  NCCL all-gather, GpuShardMode::Replicated query chunks, and k-means with an
  NCCL all-reduce of the fixed-point sums each iteration;
* one process per GPU (vrs_comm_init + vrs_knn_create_rank /
  vrs_kmeans_fit_rank), the layout torchrun launches.

kNN results must equal the single-process oracle exactly (ids and distance
bits). k-means: same iteration count, the same assignments (the GPU sums
are exact fixed-point integers, so sharding cannot change them), centroids
within 1e-6 and inertia within 1e-6 relative (the oracle sums in f64 in row
order). Mirrors ddp/distributed_knn.rs:263-360 and
ddp/distributed_kmeans.rs:544-642.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


@pytest.fixture(scope="module")
def two(vc, gpu):
    if gpu < 2:
        pytest.skip("needs 2 or more GPUs")
    return min(gpu, 8)


def _data(vc, metric, n, q, d, seed):
    kind = {COS: vc.GEN_NORMAL_UNIT, L1: vc.GEN_UNIFORM, CHEB: vc.GEN_UNIFORM,
            HELL: vc.GEN_UNIFORM_SUM1}.get(metric, vc.GEN_NORMAL)
    s = vc.config_seed(800 + seed)
    return vc.gen_rows_host(kind, s, 0, 0, n, d), vc.gen_rows_host(kind, s, 1, 0, q, d)


def _same(dg, ig, do, io):
    assert np.array_equal(ig, io), np.argwhere(ig != io)[:5]
    assert np.array_equal(dg.view(np.uint32), do.view(np.uint32))


@pytest.mark.parametrize("metric", [L2, COS, DOT, L1, HELL])
@pytest.mark.parametrize("mode", [0, 1])
def test_clique_knn(vc, orc, two, metric, mode):
    base, qs = _data(vc, metric, 40_001, 257, 64, metric)
    eng = vc.DistributedKnnEngine.try_new(base, 64, two, vc.GpuShardMode(mode),
                                          vc.DistanceMetric(metric))
    assert eng.num_gpus() == two
    for k in (1, 37, 100):
        dg, ig = eng.search_arrays(qs, k)
        do, io = orc.knn_search(base, qs, k, metric)
        _same(dg, ig, do, io)
    eng.close()


@pytest.mark.parametrize("metric,d", [(L2, 96), (L2, 128), (COS, 96), (DOT, 64)])
def test_pooled_bound_needs_no_exact_pass(vc, orc, two, metric, d):
    """Sharded tensor-core search pools the shards' pivot minima into one
    starting bound; a shard whose candidates fall short of k' certifies a
    limit in exact-score units and the merge checks it. On ordinary data no
    query may need the exact re-search (a squared-L2 limit once missed
    |q|^2 and sent every query there), and results equal the oracle's."""
    base, qs = _data(vc, metric, 300_000, 512, d, 20 + d)
    eng = vc.DistributedKnnEngine.try_new(base, d, two, vc.GpuShardMode.Sharded, vc.DistanceMetric(metric))
    vc.profile_enable(1)
    vc.profile_reset()
    try:
        dg, ig = eng.search_arrays(qs, 100)
        _, fallback_queries = vc.profile_read("knn_fallback_queries")
    finally:
        vc.profile_enable(0)
    do, io = orc.knn_search(base, qs, 100, metric)
    _same(dg, ig, do, io)
    assert fallback_queries == 0
    eng.close()


def test_clique_knn_ties_across_shards(vc, orc, two):
    """Equal rows in every shard: the merge must order equal scores by id."""
    rng = np.random.default_rng(5)
    rows = rng.standard_normal((7, 16)).astype(np.float32)
    base = np.tile(rows, (1000, 1))
    qs = rows[:3] + 0.25
    eng = vc.DistributedKnnEngine.try_new(base, 16, two, vc.GpuShardMode.Sharded,
                                          vc.DistanceMetric.L2Squared)
    dg, ig = eng.search_arrays(qs, 50)
    do, io = orc.knn_search(base, qs, 50, L2)
    _same(dg, ig, do, io)
    eng.close()


def test_more_gpus_than_rows(vc, orc, two):
    """distributed_knn.rs: fewer rows than GPUs still answers from the rows there are."""
    base, qs = _data(vc, L2, 1, 3, 8, 9)
    eng = vc.DistributedKnnEngine.try_new(base, 8, two, vc.GpuShardMode.Sharded,
                                          vc.DistanceMetric.L2Squared)
    dg, ig = eng.search_arrays(qs, 5)
    do, io = orc.knn_search(base, qs, 5, L2)
    _same(dg, ig, do, io)
    eng.close()


@pytest.mark.parametrize("metric", [L2, COS])
def test_clique_kmeans(vc, orc, two, metric):
    s = vc.config_seed(820)
    cent = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, 64, 32)
    x = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, 50_001, 32, cent, 64, 0.1)
    init = x[:64]
    res = vc.DistributedKMeansEngine.try_new(two).fit(x, 32, 64, 6, 0.0, vc.DistanceMetric(metric),
                                                      init=init)
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, 64, init, 6, 0.0, metric)
    assert res.iterations == it_o
    assert float((res.assignments == a_o).mean()) >= (1.0 if metric == L2 else 0.999)
    np.testing.assert_allclose(res.centroids, c_o, rtol=1e-6, atol=1e-6)
    assert abs(res.inertia - in_o) <= 1e-6 * abs(in_o)


# ------------------------------------------------------------ rank mode

def _rank_worker(rank, world, uid, out_q):
    sys.path.insert(0, os.path.join(ROOT, "vector-rs_b200", "python"))
    import vector_cuda as vc
    try:
        comm = vc.Comm.init(uid, world, rank, rank)
        base, qs = _data(vc, L2, 30_001, 129, 48, 40)
        r0, r1 = vc.shard_rows(len(base), world, rank)
        eng = vc.DistributedKnnEngine.create_rank(comm, base[r0:r1], 48, r0, len(base),
                                                  vc.GpuShardMode.Sharded,
                                                  vc.DistanceMetric.L2Squared)
        d, i = eng.search_arrays(qs, 64)
        # Root I/O: rank 0 alone passes queries and receives the results.
        root = eng.search_root(qs if rank == 0 else None, 64, nq=len(qs))
        ok_root = (root is None) == (rank != 0)
        if rank == 0:
            ok_root = ok_root and np.array_equal(root[1], i) and np.array_equal(root[0].view(np.uint32),
                                                                               d.view(np.uint32))
        eng.close()
        s = vc.config_seed(830)
        cent = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, 32, 24)
        x = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, 20_003, 24, cent, 32, 0.1)
        k0, k1 = vc.shard_rows(len(x), world, rank)
        res = vc.kmeans_fit_rank(comm, x[k0:k1], len(x), 24, 32, x[:32], 5, 0.0,
                                 vc.DistanceMetric.L2Squared)
        comm.close()
        out_q.put((rank, d, i, res.centroids, res.assignments, res.iterations, res.inertia, ok_root))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out_q.put((rank, "error", repr(e)))


def test_rank_mode_knn_and_kmeans(vc, orc, two):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    uid = vc.Comm.unique_id()
    procs = [ctx.Process(target=_rank_worker, args=(r, world, uid, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            item = q.get(timeout=300)
            assert not isinstance(item[1], str), item
            got[item[0]] = item
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    base, qs = _data(vc, L2, 30_001, 129, 48, 40)
    do, io = orc.knn_search(base, qs, 64, L2)
    for r in range(world):
        _same(got[r][1], got[r][2], do, io)
        assert got[r][7], f"rank {r}: root I/O search"
    s = vc.config_seed(830)
    cent = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, 32, 24)
    x = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, 20_003, 24, cent, 32, 0.1)
    c_o, a_o, it_o, in_o = orc.kmeans_fit(x, 32, x[:32], 5, 0.0, L2)
    assign = np.concatenate([got[r][4] for r in range(world)])
    assert np.array_equal(assign, a_o)
    for r in range(world):
        assert got[r][5] == it_o
        np.testing.assert_allclose(got[r][3], c_o, rtol=1e-6, atol=1e-6)
        assert abs(got[r][6] - in_o) <= 1e-6 * abs(in_o)


def test_pooled_bound_sentinel_redo(vc, orc, two):
    """Row shards pool their pivot minima into one starting bound taken at a
    rank below k; no shard can check it alone, so each cuts its merge pairs
    where its unkept rows could start (a sentinel pair). Near rows only on
    pivot rows, fewer than k of them, put a sentinel inside the merged
    top-k: the query must be searched again exactly and match the oracle."""
    n, d, k = 1_200_000, 32, 100
    rng = np.random.default_rng(12)
    qs = rng.standard_normal((3, d)).astype(np.float32)
    base = (rng.standard_normal((n, d)) * 3 + 20).astype(np.float32)
    for i in range(3):
        near = 6144 * (i * 60 + np.arange(60))  # pivot rows, 1024 pivot rows apart
        base[near] = qs[i] + 0.05 * rng.standard_normal((60, d)).astype(np.float32)
        mid = 6 * (20_000 + i * 300 + np.arange(200)) + 1
        base[mid] = qs[i] + 0.5 * rng.standard_normal((200, d)).astype(np.float32)
    eng = vc.DistributedKnnEngine.try_new(base, d, 2, vc.GpuShardMode.Sharded, vc.DistanceMetric.L2Squared)
    vc.profile_reset()
    vc.profile_enable(True)
    dg, ig = eng.search_arrays(qs, k)
    vc.profile_enable(False)
    _, n_fb = vc.profile_read("knn_fallback")
    do, io = orc.knn_search(base, qs, k, L2)
    _same(dg, ig, do, io)
    assert n_fb > 0
    eng.close()
