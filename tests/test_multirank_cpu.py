"""The multi-GPU semantics on CPU: two `gloo` ranks in child processes.

What libvrs does across GPUs, restated rank by rank with the oracle as the
per-rank compute and gloo as the collective, checked against the
single-process oracle:

* GpuShardMode::Sharded -- rows split by `shard_rows`, each rank's top-k
  with global ids (local id + r0), an all-gather, and the reference's
  top_k_reduce merge in rank order (ddp/collective.rs:115-152) give exactly
  the unsharded search, ties by lower id included;
* the same search as libvrs runs it in rank mode: queries broadcast from
  rank 0, every rank's lists exchanged so that each rank merges one slice
  of the queries, merged slices gathered on rank 0;
* GpuShardMode::Replicated -- query chunks by `query_chunk`, concatenated in
  rank order (ddp/distributed_knn.rs:201-229);
* distributed Lloyd -- per-rank assignment, sums and counts, an all-reduce,
  and the shared update (ddp/distributed_kmeans.rs:377-461) give the
  single-process fit;
* a rank that exits without joining a collective makes the survivor's
  collective fail with an error inside its timeout instead of hanging.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (os.path.join(ROOT, "vector-rs_b200", "python"), os.path.join(ROOT, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _init(rank, world, port, seconds=60):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=seconds))
    return dist


def _knn_data(vc, metric, n, q, d, seed):
    s = vc.config_seed(700 + seed)
    kind = vc.GEN_UNIFORM if metric in (L1, CHEB, HAM) else vc.GEN_NORMAL
    base = vc.gen_rows_host(kind, s, 0, 0, n, d)
    qs = vc.gen_rows_host(kind, s, 1, 0, q, d)
    if metric == HAM:  # coarse values: many equal distances across the shard boundary
        base, qs = np.round(base * 2) / 2, np.round(qs * 2) / 2
    return np.ascontiguousarray(base, np.float32), np.ascontiguousarray(qs, np.float32)


def _sharded_knn(rank, world, port, out_q):
    _paths()
    import oracle
    import vector_cuda as vc
    dist = _init(rank, world, port)
    ok = True
    for metric in (L2, DOT, COS, L1, HAM):
        n = 1001  # ceil(1001 / 2) = 501: unequal shards
        base, qs = _knn_data(vc, metric, n, 13, 9, metric)
        r0, r1 = vc.shard_rows(n, world, rank)
        for k in (1, 7, 40):
            d_loc, i_loc = oracle.knn_search(base[r0:r1], qs, k, metric, nthreads=2)
            i_loc = i_loc + np.uint32(r0)
            gathered = [None] * world
            dist.all_gather_object(gathered, (d_loc, i_loc))
            if rank == 0:
                d_full, i_full = oracle.knn_search(base, qs, k, metric, nthreads=2)
                for qi in range(len(qs)):
                    md, mi = oracle.topk_reduce([(g[0][qi], g[1][qi]) for g in gathered], k, metric)
                    ok &= bool(np.array_equal(mi, i_full[qi]))
                    ok &= bool(np.array_equal(md.view(np.uint32), d_full[qi].view(np.uint32)))
    if rank == 0:
        out_q.put(("sharded", ok))
    dist.destroy_process_group()


def _sliced_merge_knn(rank, world, port, out_q):
    """The merge protocol of a row-sharded search in rank mode: rank 0 alone
    holds the queries and broadcasts them; each rank's top-k' lists (global
    ids) are padded to world * c rows (c = ceil(nq / world)) and exchanged so
    that rank p holds every rank's lists for queries [p c, (p+1) c); rank p
    merges that slice in rank order; the merged slices are gathered on rank
    0 alone. The result must be the unsharded search."""
    _paths()
    import torch
    import oracle
    import vector_cuda as vc
    dist = _init(rank, world, port)
    ok = True
    for metric, n, nq in ((L2, 1001, 13), (COS, 640, 8), (HAM, 999, 5)):
        base, qs_all = _knn_data(vc, metric, n, nq, 9, 20 + metric)
        k = 7
        q = torch.from_numpy(qs_all.copy()) if rank == 0 else torch.zeros((nq, 9), dtype=torch.float32)
        dist.broadcast(q, src=0)
        qs = q.numpy()
        r0, r1 = vc.shard_rows(n, world, rank)
        d_loc, i_loc = oracle.knn_search(base[r0:r1], qs, k, metric, nthreads=2)
        c = -(-nq // world)
        pad_d = np.full((world * c, k), np.nan, np.float32)
        pad_i = np.full((world * c, k), 0xFFFFFFFF, np.uint32)
        pad_d[:nq], pad_i[:nq] = d_loc, i_loc + np.uint32(r0)
        recv_d = torch.empty((world * c, k), dtype=torch.float32)
        recv_i = torch.empty((world * c, k), dtype=torch.int64)
        dist.all_to_all_single(recv_d, torch.from_numpy(pad_d))
        dist.all_to_all_single(recv_i, torch.from_numpy(pad_i.astype(np.int64)))
        rd, ri = recv_d.numpy().reshape(world, c, k), recv_i.numpy().reshape(world, c, k).astype(np.uint32)
        md = np.full((c, k), np.nan, np.float32)
        mi = np.full((c, k), 0xFFFFFFFF, np.uint32)
        for j in range(c):
            if rank * c + j >= nq:
                continue  # padding query
            lists = [(rd[g, j], ri[g, j]) for g in range(world)]
            dd, ii = oracle.topk_reduce(lists, k, metric)
            md[j, :len(dd)], mi[j, :len(ii)] = dd, ii
        slices = [None] * world
        dist.all_gather_object(slices, (md, mi))
        if rank == 0:
            gd = np.concatenate([x[0] for x in slices])[:nq]
            gi = np.concatenate([x[1] for x in slices])[:nq]
            d_full, i_full = oracle.knn_search(base, qs_all, k, metric, nthreads=2)
            ok &= bool(np.array_equal(gi, i_full))
            ok &= bool(np.array_equal(gd.view(np.uint32), d_full.view(np.uint32)))
    if rank == 0:
        out_q.put(("sliced", ok))
    dist.destroy_process_group()


def _replicated_knn(rank, world, port, out_q):
    _paths()
    import oracle
    import vector_cuda as vc
    dist = _init(rank, world, port)
    base, qs = _knn_data(vc, L2, 500, 21, 16, 3)  # 21 queries: chunks of 11 and 10
    q0, q1 = vc.query_chunk(len(qs), world, rank)
    d_loc, i_loc = oracle.knn_search(base, qs[q0:q1], 10, L2, nthreads=2)
    gathered = [None] * world
    dist.all_gather_object(gathered, (d_loc, i_loc))
    if rank == 0:
        d_full, i_full = oracle.knn_search(base, qs, 10, L2, nthreads=2)
        ok = np.array_equal(np.concatenate([g[1] for g in gathered]), i_full)
        ok &= np.array_equal(np.concatenate([g[0] for g in gathered]), d_full)
        out_q.put(("replicated", bool(ok)))
    dist.destroy_process_group()


def _distributed_lloyd(rank, world, port, out_q):
    _paths()
    import torch
    import oracle
    import vector_cuda as vc
    dist = _init(rank, world, port)
    s = vc.config_seed(710)
    n, d, K, iters = 3001, 12, 6, 9
    cent = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, K, d)
    x = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, n, d, cent, K, 0.4)
    init = np.ascontiguousarray(x[:K])
    r0, r1 = vc.shard_rows(n, world, rank)
    ok = True
    for metric in (L2, COS):
        c = init.copy()
        assign_loc, inertia = None, 0.0
        it = 0
        for it in range(1, iters + 1):
            assign_loc, sums, counts, inertia_loc = oracle.kmeans_local(x[r0:r1], c, metric,
                                                                        nthreads=2)
            ts, tc = torch.from_numpy(sums), torch.from_numpy(counts)
            ti = torch.tensor([inertia_loc], dtype=torch.float64)
            dist.all_reduce(ts)
            dist.all_reduce(tc)
            dist.all_reduce(ti)
            inertia = float(ti.item())
            if oracle.kmeans_update(ts.numpy(), tc.numpy(), c) <= 0.0:
                break
        gathered = [None] * world
        dist.all_gather_object(gathered, assign_loc)
        if rank == 0:
            c_o, a_o, it_o, in_o = oracle.kmeans_fit(x, K, init, iters, 0.0, metric, nthreads=2)
            ok &= it == it_o
            ok &= bool(np.array_equal(np.concatenate(gathered), a_o))
            ok &= bool(np.allclose(c, c_o, rtol=1e-6, atol=1e-7))
            ok &= abs(inertia - in_o) <= 1e-9 * abs(in_o)
    if rank == 0:
        out_q.put(("lloyd", ok))
    dist.destroy_process_group()


def _early_exit(rank, world, port, out_q):
    _paths()
    import torch
    dist = _init(rank, world, port, seconds=3)
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks take the first step
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    try:
        dist.all_reduce(t)
        out_q.put(("early_exit", False))
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        out_q.put(("early_exit", "error:" + type(e).__name__))
    out_q.close()
    out_q.join_thread()  # flush the result before the hard exit
    os._exit(0)


def _run(fn, timeout=240):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=timeout)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.parametrize("fn,name", [(_sharded_knn, "sharded"), (_sliced_merge_knn, "sliced"),
                                     (_replicated_knn, "replicated"), (_distributed_lloyd, "lloyd")])
def test_two_rank_semantics(fn, name):
    got = _run(fn)
    assert got == (name, True)


def test_rank_that_leaves_fails_the_next_collective():
    name, res = _run(_early_exit, timeout=120)
    assert name == "early_exit" and isinstance(res, str) and res.startswith("error:"), res
