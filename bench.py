#!/usr/bin/env python
"""bench.py -- flat kNN queries/s (default C2: 1M x 128 cosine, k=100) and
k-means iterations/s (default C3) on B200, through libvrs's C ABI.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c4-l1|c4-linf|c4-hell|c5a] [--km-workload c3|c5b]
                    [--no-scale] [--km-parity-iters I]

N > 1 is launched by torchrun (one process per GPU); each rank holds a row
shard of the base (GpuShardMode::Sharded) and the ranks meet in NCCL
collectives and a GPU merge inside vrs_knn_search. Prints one JSON line on
rank 0.

A step is one vrs_knn_search of the 10,000 C2 queries against the whole
(sharded) 1,000,000 x 128 base. `value` times steps whose queries and
results stay in HBM; `e2e` times the same call with pinned host buffers
(H2D of the queries and D2H of the results inside the timed region);
`sustained` repeats the step for at least a second under its own clock
record. The base (512 MB of f32) is larger than L2, so no flush is needed
between steps. Inputs are seeded Philox4x32-10 draws generated on the
device, the same bits the CPU oracle consumes. At every N rank 0 checks a
query sample of the merged results, and a k-means fit of the same init,
against the oracle on the whole base. The north star's scale configs (C5a:
100M x 96 squared-L2 kNN; C5b: 10M x 96, K = 16384 k-means) ride along as
the keys `c5a` and `c5b`.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vector-rs_b200", "python"))

import numpy as np  # noqa: E402

L2, DOT, COS, L1, CHEB, HELL = 0, 1, 2, 3, 5, 9

# kNN workloads (the default is the headline C2).
# seed index = config index (C1 0, C2 1, C3 2, C4 3, C5 4).
WORKLOADS = {
    "c2": dict(metric=COS, n=1_000_000, d=128, nq=10_000, k=100, gen="GEN_NORMAL_UNIT", seed=1,
               cpu_sample=1000,
               name="C2 cosine flat kNN: base 1,000,000 x 128, 10,000 queries, k=100, "
                    "GpuShardMode::Sharded over N GPUs",
               data="synthetic: Philox4x32-10 N(0,1) rows L2-normalised (f64), generated on device"),
    "c1": dict(metric=L2, n=10_000, d=128, nq=1_000, k=10, gen="GEN_NORMAL", seed=0, cpu_sample=1000,
               name="C1 squared-L2 flat kNN: base 10,000 x 128, 1,000 queries, k=10",
               data="synthetic: Philox4x32-10 N(0,1), generated on device"),
    "c4-l1": dict(metric=L1, n=1_000_000, d=96, nq=10_000, k=10, gen="GEN_UNIFORM", seed=3, cpu_sample=200,
                  name="C4 Manhattan flat kNN: base 1,000,000 x 96 U[0,1), 10,000 queries, k=10",
                  data="synthetic: Philox4x32-10 U[0,1), generated on device"),
    "c4-linf": dict(metric=CHEB, n=1_000_000, d=96, nq=10_000, k=10, gen="GEN_UNIFORM", seed=3, cpu_sample=200,
                    name="C4 Chebyshev flat kNN: base 1,000,000 x 96 U[0,1), 10,000 queries, k=10",
                    data="synthetic: Philox4x32-10 U[0,1), generated on device"),
    "c4-hell": dict(metric=HELL, n=1_000_000, d=96, nq=10_000, k=10, gen="GEN_UNIFORM_SUM1", seed=3,
                    cpu_sample=200,
                    name="C4 Hellinger flat kNN: base 1,000,000 x 96 U[0,1) rows scaled to sum 1, "
                         "10,000 queries, k=10",
                    data="synthetic: Philox4x32-10 U[0,1) rows scaled to sum 1 (f64), generated on device"),
    "c5a": dict(metric=L2, n=100_000_000, d=96, nq=10_000, k=100, gen="GEN_NORMAL", seed=4, cpu_sample=20,
                name="C5a squared-L2 flat kNN: base 100,000,000 x 96 N(0,1) (38.4 GB), 10,000 queries, "
                     "k=100, row-sharded",
                data="synthetic: Philox4x32-10 N(0,1), generated on device shard by shard"),
}
# k-means workloads (the default is C3).
KM_WORKLOADS = {
    "c3": dict(n=1_000_000, d=128, K=1024, iters=20, sigma=0.1, seed=2, stream_c=2, stream_x=0,
               name="C3: 1M x 128, K=1024, 20 iterations"),
    "c5b": dict(n=10_000_000, d=96, K=16_384, iters=10, sigma=0.05, seed=4, stream_c=5, stream_x=6,
                name="C5b: 10M x 96, K=16384, 10 iterations"),
}
METRIC_NAMES = {L2: "squared-L2", DOT: "dot", COS: "cosine", L1: "Manhattan", CHEB: "Chebyshev",
                HELL: "Hellinger"}
TC_METRICS = (L2, DOT, COS, 7)
# DRAM bytes (read + write) of one candidate-scan launch (the pair kernel)
# over the full C2 base, from the ncu capture summarised in
# profiles/knn_scan_tc2_C2.txt; other base sizes scale it by the rows scanned
# (the traffic is the base re-stream plus the candidate lists, both
# proportional to the rows).
SCAN_DRAM_BYTES_C2 = 382.762752e6 + 36.893184e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--km-workload", choices=sorted(KM_WORKLOADS), default="c3")
    ap.add_argument("--no-kmeans", action="store_true")
    ap.add_argument("--no-knn", action="store_true", help="k-means only (its line becomes the output)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--ivf", action="store_true",
                    help="IVF coarse probe/assign line only (1 GPU; not part of the default run)")
    ap.add_argument("--ivfpq", action="store_true",
                    help="IVF-PQ ADC search line only (1 GPU; not part of the default run)")
    ap.add_argument("--storage", action="store_true",
                    help="VECRSTOR file -> GPU engine load line only (1 GPU; not part of the default run)")
    ap.add_argument("--n-base", type=int, default=None, help="override the workload's base rows")
    ap.add_argument("--n-query", type=int, default=None, help="override the workload's query count")
    ap.add_argument("--km-n", type=int, default=None, help="override the k-means point count")
    ap.add_argument("--km-iters", type=int, default=None)
    ap.add_argument("--km-parity-iters", type=int, default=2,
                    help="Lloyd iterations of the k-means oracle comparison on all points (0: skip)")
    ap.add_argument("--no-scale", action="store_true",
                    help="skip the north-star scale configs (C5a kNN, C5b k-means) that ride along as keys")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during a timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # The timed region is short: start it only once samples flow.
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def host_gen(vc, kind, seed, stream, rows, d, threads=None):
    """Host copy of generator rows from the product library, in parallel chunks."""
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty((rows, d), np.float32)
    nt = threads or os.cpu_count() or 1
    chunk = max(1, -(-rows // (nt * 4)))

    def work(r0):
        n = min(chunk, rows - r0)
        out[r0:r0 + n] = vc.gen_rows_host(kind, seed, stream, r0, n, d)

    with ThreadPoolExecutor(nt) as ex:
        list(ex.map(work, range(0, rows, chunk)))
    return out


def oracle_mod():
    """The CPU oracle (restated reference CPU path): the parity checker and
    the CPU baseline, never the measured GPU path."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    return oracle


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def workload(args):
    w = dict(WORKLOADS[args.workload])
    if args.n_base:
        w["n"] = args.n_base
    if args.n_query:
        w["nq"] = args.n_query
    return w


def km_workload(args, name=None):
    w = dict(KM_WORKLOADS[name or args.km_workload])
    if name is None:
        if args.km_n:
            w["n"] = args.km_n
        if args.km_iters:
            w["iters"] = args.km_iters
    return w


def fmt_count(n):
    if n % 1_000_000 == 0:
        return f"{n // 1_000_000}M"
    if n % 1000 == 0:
        return f"{n // 1000}k"
    return str(n)


def metric_label(w):
    return f"flat kNN queries/s ({fmt_count(w['n'])} x {w['d']} {METRIC_NAMES[w['metric']]}, k={w['k']})"


def knn_config(w, world):
    n_loc = -(-w["n"] // world)
    big = n_loc * w["d"] * 4 > 126e6
    return {"workload": w["name"], "n_base": w["n"], "queries_per_step": w["nq"], "k": w["k"], "dim": w["d"],
            "parallelism": f"row-sharded x{world}; queries broadcast from rank 0, per-query-slice "
                           "NCCL exchange + GPU merge, results to rank 0",
            "l2": ("inputs larger than L2 (f32 base shard %.0f MB), no flush" % (n_loc * w["d"] * 4 / 1e6))
                  if big else "base shard smaller than L2: steps see a warm L2"}


def parity_stats(gd, gi, od, oi):
    """Per-position comparison with the oracle: ids, distance bits, and the
    largest relative distance error (the north star allows 1e-4)."""
    gd, od = np.asarray(gd, np.float32), np.asarray(od, np.float32)
    den = np.maximum(np.abs(od.astype(np.float64)), 1.0)
    rel = np.abs(gd.astype(np.float64) - od.astype(np.float64)) / den
    return {"queries": int(len(gi)), "ids_equal_frac": float((np.asarray(gi) == np.asarray(oi)).mean()),
            "dist_bit_equal_frac": float((gd.view(np.uint32) == od.view(np.uint32)).mean()),
            "max_rel_dist_err": float(rel.max()) if rel.size else 0.0}


def oracle_topk_streamed(orc, vc, torch, dev, w, seed, kind, q_host, chunk_rows=2_000_000):
    """Oracle top-k of a few queries over a base too large for one host copy:
    rows are generated on this GPU chunk by chunk (the same bits the shards
    hold), copied to pinned host memory and searched by the row-split oracle
    with global ids; the per-chunk lists merge per query in (score, id)
    order. Squared L2, dot and cosine only (their reported values order
    like the ranking key)."""
    n, D, K, metric = w["n"], w["d"], w["k"], w["metric"]
    assert metric in (L2, DOT, COS)
    sign = -1.0 if metric in (DOT, COS) else 1.0
    rows = min(chunk_rows, n)
    buf = torch.empty((rows, D), dtype=torch.float32, device=dev)
    pin = torch.empty((rows, D), dtype=torch.float32, pin_memory=True)
    run_d = run_i = None
    for r0 in range(0, n, rows):
        rc = min(rows, n - r0)
        vc.gen_rows_device(kind, seed, 0, r0, rc, D, buf.data_ptr())
        torch.cuda.synchronize(dev)
        pin[:rc].copy_(buf[:rc])
        d, i = orc.knn_search_rows(pin[:rc].numpy(), q_host, K, metric, nthreads=host_cores(), id_offset=r0)
        if run_d is None:
            run_d, run_i = d.copy(), i.copy()
            continue
        cd = np.concatenate([run_d, d], 1)
        ci = np.concatenate([run_i, i], 1)
        for r in range(cd.shape[0]):
            o = np.lexsort((ci[r].astype(np.int64), sign * cd[r].astype(np.float64)))[:K]
            run_d[r], run_i[r] = cd[r][o], ci[r][o]
    del buf
    return run_d, run_i


def reference_arm(args):
    """The reference's CPU path (the oracle's restatement of
    search_batch_cpu, all host threads) on the same workload, a bounded query
    sample per step; inputs from the oracle's own generator (the same bits
    as the GPU arm's), so this process never loads libvrs. Also times the
    restated fit_cpu for one Lloyd iteration of the k-means config."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    orc = oracle_mod()
    cores = host_cores()
    w = workload(args)
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    seed = orc.config_seed(w["seed"])
    kind = getattr(orc, w["gen"])
    base = orc.gen_rows(kind, seed, 0, 0, w["n"], w["d"], nthreads=cores)
    queries = orc.gen_rows(kind, seed, 1, 0, min(w["nq"], 2000), w["d"], nthreads=cores)
    per_step = max(1, min(100, w["cpu_sample"]))
    for _ in range(args.warmup):
        orc.knn_search(base, queries[:16], w["k"], w["metric"], nthreads=cores)
    t0 = time.perf_counter()
    for s in range(args.steps):
        q0 = (s * per_step) % (len(queries) - per_step + 1)
        orc.knn_search(base, queries[q0:q0 + per_step], w["k"], w["metric"], nthreads=cores)
    dt = time.perf_counter() - t0
    v = per_step * args.steps / dt
    sample = (f"{per_step} of the {w['nq']} queries per step against the full {w['n']}-row base, "
              f"{cores} threads (the reference's Rust cannot build here: no cargo; oracle restatement "
              "of search_batch_cpu)")
    line = {
        "impl": "reference", "metric": metric_label(w), "value": v,
        "unit": "queries/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": w["data"].replace("generated on device", "host"),
        "config": knn_config(w, world), "sample": sample,
        "cpu_baseline": {"value": v, "unit": "queries/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    del base
    if not args.no_kmeans:
        kw = km_workload(args)
        ks = orc.config_seed(kw["seed"])
        cent = orc.gen_rows(orc.GEN_NORMAL, ks, kw["stream_c"], 0, kw["K"], kw["d"])
        x = orc.gen_rows(orc.GEN_MIXTURE, ks, kw["stream_x"], 0, kw["n"], kw["d"], cent, kw["K"], kw["sigma"],
                         nthreads=cores)
        t0 = time.perf_counter()
        _, _, it, _ = orc.kmeans_fit(x, kw["K"], x[:kw["K"]], 1, 0.0, L2, nthreads=cores)
        ks_dt = time.perf_counter() - t0
        line["kmeans"] = {"metric": f"k-means iterations/s ({kw['name']})", "value": it / ks_dt,
                          "unit": "iterations/s", "cores": cores, "kind": "port",
                          "sample": f"{it} Lloyd iteration(s) of the {kw['iters']} on all {kw['n']} points "
                                    "(oracle restatement of fit_cpu)"}
    print(json.dumps(line), flush=True)
    return 0


class Ctx:
    """Per-process bench state shared by the workload runners."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    import vector_cuda as vc

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    uid = [vc.Comm.unique_id() if rank == 0 else None]
    if dist:
        dist.broadcast_object_list(uid, src=0)
    comm = vc.Comm.init(uid[0], world, rank, local)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_rows(t):
        """Rank-ordered concatenation of every rank's rows (rank 0 uses it)."""
        if not dist:
            return t
        n = torch.tensor([t.shape[0]], dtype=torch.int64, device=dev)
        ns = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(ns, n)
        m = int(max(x.item() for x in ns))
        pad = torch.zeros((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
        pad[:t.shape[0]] = t
        outs = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(outs, pad)
        return torch.cat([o[:int(c.item())] for o, c in zip(outs, ns)])

    pk, pk_kind = peaks()
    ctx = Ctx(args=args, vc=vc, torch=torch, comm=comm, dev=dev, world=world, rank=rank, local=local,
              stream=stream, barrier=barrier, max_over_ranks=max_over_ranks, gather_rows=gather_rows,
              pk=pk, pk_kind=pk_kind, peak_burst=pk.get("bf16_tflops", 1590.0),
              peak_sus=pk.get("bf16_tflops_sustained", pk.get("bf16_tflops", 1400.0)))
    line = None
    if args.ivf:
        line = ivf_bench(args, vc, torch, dev, ctx.peak_burst) if rank == 0 else None
        args.no_knn = args.no_kmeans = True
    if args.storage:
        line = storage_bench(args, vc, torch, dev, pk) if rank == 0 else None
        args.no_knn = args.no_kmeans = True
    if args.ivfpq:
        line = ivfpq_bench(args, vc, torch, dev, pk, pk_kind) if rank == 0 else None
        args.no_knn = args.no_kmeans = True
    if not args.no_knn:
        w = workload(args)
        line = knn_bench(ctx, w, args.steps, args.warmup, parity_queries=min(w["cpu_sample"], w["nq"]),
                         cpu_leg=not args.no_cpu, sustained=True)
    if not args.no_kmeans:
        km = kmeans_bench(ctx, km_workload(args), parity_iters=args.km_parity_iters, cpu_leg=not args.no_cpu)
        if line is None:
            line = km
        else:
            line["kmeans"] = km
    # The north star's scale configs ride along as extra keys of the default
    # line (few steps each), so every scaling run records them too.
    if line is not None and not args.no_scale and not args.ivf and not args.storage and not args.ivfpq:
        c5a = dict(WORKLOADS["c5a"])
        line["c5a"] = knn_bench(ctx, c5a, min(args.steps, 5), min(args.warmup, 2), parity_queries=20,
                                cpu_leg=False, sustained=False, e2e_steps=2)
        line["c5b"] = kmeans_bench(ctx, km_workload(args, "c5b"), parity_iters=1, cpu_leg=False,
                                   parity_sample=20_000, sustained=False, e2e=False)
    comm.close()
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def knn_bench(ctx, w, steps, warmup, parity_queries, cpu_leg, sustained, e2e_steps=None):
    vc, torch, dev, world, rank = ctx.vc, ctx.torch, ctx.dev, ctx.world, ctx.rank
    stream, barrier, max_over_ranks = ctx.stream, ctx.barrier, ctx.max_over_ranks
    n_base, n_q, D, K, metric = w["n"], w["nq"], w["d"], w["k"], w["metric"]
    seed = vc.config_seed(w["seed"])
    kind = getattr(vc, w["gen"])
    r0, r1 = vc.shard_rows(n_base, world, rank)
    n_loc = r1 - r0
    shard = torch.empty((max(n_loc, 1), D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(kind, seed, 0, r0, n_loc, D, shard.data_ptr())
    q_dev = torch.empty((n_q, D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(kind, seed, 1, 0, n_q, D, q_dev.data_ptr())
    torch.cuda.synchronize()
    eng = vc.DistributedKnnEngine.create_rank(ctx.comm, None, D, r0, n_base, vc.GpuShardMode.Sharded,
                                              vc.DistanceMetric(metric),
                                              device_ptr=shard.data_ptr(), n_local=n_loc)
    eng.set_stream(stream.cuda_stream)
    keep_shard = world == 1 and n_base * D * 4 <= 4e9 and rank == 0  # host copy for the oracle
    base_h = shard[:n_loc].cpu().numpy() if keep_shard else None
    del shard  # the engine holds its own padded copy
    torch.cuda.empty_cache()
    out_d = torch.empty((n_q, K), dtype=torch.float32, device=dev)
    out_i = torch.empty((n_q, K), dtype=torch.int32, device=dev)

    # Root I/O: rank 0 alone supplies the queries (broadcast to the other
    # ranks over NVLink) and receives the merged results, like the one
    # caller of search_batch; the other ranks pass no buffers.
    root = rank == 0

    def step_dev():
        return eng.search_device(q_dev.data_ptr() if root else 0, n_q, K, out_d.data_ptr() if root else 0,
                                 out_i.data_ptr() if root else 0, root=True)

    for _ in range(warmup):
        step_dev()
    barrier()
    vc.profile_reset()  # the launch counter covers the timed steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(ctx.local) as clk:
        barrier()
        ev0.record(stream)
        for _ in range(steps):
            step_dev()
        ev1.record(stream)
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    launches = vc.profile_read("*")[1]
    # Results of the timed steps (on rank 0), for the parity check.
    res_i = out_i.cpu().numpy().view(np.uint32).copy() if rank == 0 else None
    res_d = out_d.cpu().numpy().copy() if rank == 0 else None
    # Per-kernel breakdown from the same steps run again with the library's
    # CUDA-event profiling on (its events cost host time per launch, so the
    # timed loop above runs without it).
    vc.profile_reset()
    vc.profile_enable(True)
    for _ in range(steps):
        step_dev()
    barrier()
    vc.profile_enable(False)
    st = {nm: vc.profile_read(nm) for nm in ("knn_scan", "knn_select", "knn_merge", "knn_pivot", "knn_fallback",
                                             "knn_prep", "knn_gather", "knn_fallback_queries")}
    value = n_q * steps / (ms / 1e3)

    # Sustained: the same step repeated for at least one second (its own
    # clock record), so the clocks seen under a longer load are on file.
    sus = None
    if sustained:
        n_sus = max(steps, int(np.ceil(1000.0 / max(ms / steps, 1e-3))))
        n_sus = int(max_over_ranks(float(n_sus)))
        with ClockSampler(ctx.local) as clk_s:
            barrier()
            ev0.record(stream)
            for _ in range(n_sus):
                step_dev()
            ev1.record(stream)
            barrier()
        ms_s = max_over_ranks(ev0.elapsed_time(ev1))
        sus = {"steps": n_sus, "seconds": ms_s / 1e3, "value": n_q * n_sus / (ms_s / 1e3),
               "ms_per_step": ms_s / n_sus, "clocks": clk_s.summary()}

    # ----------------------------------------------------------- e2e (host)
    q_host = torch.empty((n_q, D), dtype=torch.float32, pin_memory=True)
    q_host.copy_(q_dev.cpu())
    hd = torch.empty((n_q, K), dtype=torch.float32, pin_memory=True)
    hi = torch.empty((n_q, K), dtype=torch.int32, pin_memory=True)

    def step_host():
        kk = vc.ctypes.c_int32()
        vp = (lambda t: vc.ctypes.c_void_p(t.data_ptr())) if root else (lambda t: None)
        vc._check(vc.lib().vrs_knn_search_ex(eng._h, vp(q_host), n_q, K, vp(hd), vp(hi), vc.ctypes.byref(kk),
                                            vc.MEM_ROOT))

    ne = e2e_steps or steps
    for _ in range(max(1, warmup // 2)):
        step_host()
    with ClockSampler(ctx.local) as clk2:
        # Ranks meet after their samplers start, so no rank's first
        # collective waits out another rank's sampler start-up.
        barrier()
        ev0.record(stream)
        for _ in range(ne):
            step_host()
        ev1.record(stream)
        barrier()
    ms_e2e = max_over_ranks(ev0.elapsed_time(ev1))
    e2e = n_q * ne / (ms_e2e / 1e3)

    # ------------------------------------------------------------- roofline
    scan_ms, scan_n = st["knn_scan"]
    per_launch_ms = scan_ms / max(scan_n, 1)
    breakdown = {k.replace("knn_", ""): v[0] / steps for k, v in st.items() if k != "knn_fallback_queries"}
    breakdown["fallback_launches"] = st["knn_fallback"][1]
    breakdown["fallback_queries_per_step"] = st["knn_fallback_queries"][1] / steps
    if metric in TC_METRICS and D <= 128:
        flops_per_launch = 2.0 * n_loc * D * n_q  # algorithmic: 2*N_local*D per query
        achieved = flops_per_launch / (per_launch_ms / 1e3) / 1e12
        is_c2 = w["name"] == WORKLOADS["c2"]["name"] and n_base == WORKLOADS["c2"]["n"] and \
            n_q == WORKLOADS["c2"]["nq"]
        roofline = {"bound": "tensor", "kernel": "knn_scan", "achieved": achieved, "peak": ctx.peak_burst,
                    "unit": "TFLOP/s", "frac": achieved / ctx.peak_burst,
                    "peak_source": f"{ctx.pk_kind} bf16 dense, burst (the scan is timed in a short region)",
                    "frac_of_sustained": achieved / ctx.peak_sus,
                    "per_launch_ms": per_launch_ms, "launches": scan_n,
                    "flops_per_launch": flops_per_launch,
                    "traffic": SCAN_DRAM_BYTES_C2 * n_loc / n_base if is_c2 else None,
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one full-size "
                                      "C2 launch, scaled by rows scanned per GPU" if is_c2 else None,
                    "breakdown_ms_per_step": breakdown,
                    "note": "knn_scan = tcgen05 fp16 distance GEMM fused with thresholded candidate "
                            "lists (pivot-seeded bound); survivors re-ranked exactly in f32"}
        dtype = "fp16 tensor-core scan (f32 accumulate) + f32 exact re-rank"
    else:
        bytes_per_launch = n_loc * D * 4.0 + n_q * D * 4.0 + n_q * K * 8.0
        gbs = bytes_per_launch / (per_launch_ms / 1e3) / 1e9
        ops = 2.0 * n_loc * D * n_q
        clock_mhz = clk.summary().get("sm_mhz") or 1965.0
        fp32_peak = 148 * 128 * clock_mhz * 1e6 / 1e12  # FP32 lanes x clock, T ops/s
        ach_ops = ops / (per_launch_ms / 1e3) / 1e12
        roofline = {"bound": "hbm", "kernel": "knn_scan", "achieved": gbs, "peak": ctx.pk["hbm_gbs"],
                    "unit": "GB/s", "frac": gbs / ctx.pk["hbm_gbs"], "peak_source": f"{ctx.pk_kind} HBM copy",
                    "per_launch_ms": per_launch_ms, "launches": scan_n,
                    "bytes_per_launch": bytes_per_launch, "traffic": None,
                    "binding": {"pipe": "fp32 CUDA cores", "achieved": ach_ops, "unit": "T ops/s",
                                "peak": fp32_peak, "frac": ach_ops / fp32_peak,
                                "ops_per_launch": ops,
                                "peak_source": "148 SMs x 128 FP32 lanes x median SM clock in the timed region"},
                    "breakdown_ms_per_step": breakdown,
                    "note": "knn_scan = register-blocked CUDA-core scan (2 FP32 ops per element pair) "
                            "with pivot-seeded bounds; survivors re-ranked exactly"}
        dtype = "f32 CUDA-core scan + f32 exact re-rank"
    line = {
        "metric": metric_label(w), "value": value,
        "unit": "queries/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dtype, "data": w["data"],
        "config": knn_config(w, world),
        "roofline": roofline,
        "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": n_q * D * 4,
                "d2h_bytes_per_step": n_q * K * 8, "ms_per_step": ms_e2e / ne, "steps": ne},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
        "clocks_e2e": clk2.summary(),
    }
    if sus:
        line["sustained"] = sus
    del q_host, hd, hi
    eng.close()
    torch.cuda.empty_cache()

    # ------------------------------------- parity (every N) and CPU baseline
    # Rank 0 checks the merged results of the timed steps against the
    # oracle on the whole base; the other ranks wait at the barrier.
    if rank == 0 and parity_queries > 0:
        orc = oracle_mod()
        cores = host_cores()
        sample = min(parity_queries, n_q)
        q_h = q_dev[:sample].cpu().numpy()
        if base_h is None and n_base * D * 4 <= 4e9:
            full = torch.empty((n_base, D), dtype=torch.float32, device=dev)
            vc.gen_rows_device(kind, seed, 0, 0, n_base, D, full.data_ptr())
            torch.cuda.synchronize()
            base_h = full.cpu().numpy()
            del full
        if base_h is not None:
            t0 = time.perf_counter()
            do, io = orc.knn_search(base_h, q_h, K, metric, nthreads=cores)
            dt = time.perf_counter() - t0
            how = "oracle knn_search over the whole base (host copy)"
        else:
            t0 = time.perf_counter()
            do, io = oracle_topk_streamed(orc, vc, torch, dev, w, seed, kind, q_h)
            dt = time.perf_counter() - t0
            how = "oracle over the whole base, regenerated chunk by chunk on GPU 0 and merged by (score, id)"
        line["parity_sample"] = dict(parity_stats(res_d[:sample], res_i[:sample], do, io), how=how,
                                     n_gpus=world)
        if cpu_leg and world == 1 and base_h is not None:
            line["cpu_baseline"] = {
                "value": sample / dt, "unit": "queries/s", "cores": cores, "kind": "port",
                "sample": f"{sample} of the {n_q} queries against the full {n_base}-row base "
                          f"(AVX-512 restatement of search_batch_cpu, {cores} threads)",
                "seconds": dt}
        torch.cuda.empty_cache()
    del q_dev, base_h
    barrier()
    return line


def kmeans_bench(ctx, w, parity_iters, cpu_leg, parity_sample=None, sustained=True, e2e=True):
    vc, torch, dev, world, rank = ctx.vc, ctx.torch, ctx.dev, ctx.world, ctx.rank
    barrier, max_over_ranks = ctx.barrier, ctx.max_over_ranks
    KMN, KM_D, KM_K = w["n"], w["d"], w["K"]
    km_seed = vc.config_seed(w["seed"])
    k0, k1 = vc.shard_rows(KMN, world, rank)
    n_loc = k1 - k0
    cent = torch.empty((KM_K, KM_D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_NORMAL, km_seed, w["stream_c"], 0, KM_K, KM_D, cent.data_ptr())
    xs = torch.empty((max(n_loc, 1), KM_D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_MIXTURE, km_seed, w["stream_x"], k0, n_loc, KM_D, xs.data_ptr(),
                       cent.data_ptr(), KM_K, w["sigma"])
    init = torch.empty((KM_K, KM_D), dtype=torch.float32, device=dev)  # the first K points
    vc.gen_rows_device(vc.GEN_MIXTURE, km_seed, w["stream_x"], 0, KM_K, KM_D, init.data_ptr(),
                       cent.data_ptr(), KM_K, w["sigma"])
    init_h = init.cpu().numpy()
    torch.cuda.synchronize()
    M = vc.DistanceMetric.L2Squared

    def fit(iters):
        return vc.kmeans_fit_rank(ctx.comm, None, KMN, KM_D, KM_K, init_h, iters, 0.0, M,
                                  device_ptr=xs.data_ptr(), n_local=n_loc)

    fit(2)
    barrier()
    # Timed fit: only the whole Lloyd loop is bracketed by events (per-stage
    # events would add host work to every iteration).
    vc.profile_reset()
    vc.profile_enable(2)
    with ClockSampler(ctx.local) as clk:
        barrier()
        t0 = time.perf_counter()
        res = fit(w["iters"])
        barrier()
        km_s = max_over_ranks(time.perf_counter() - t0)
    vc.profile_enable(False)
    loop_ms, _ = vc.profile_read("kmeans_loop")
    loop_s = max_over_ranks(loop_ms / 1e3)
    # Per-stage breakdown from the same fit run again with every stage timed.
    barrier()
    vc.profile_reset()
    vc.profile_enable(True)
    fit(w["iters"])
    barrier()
    vc.profile_enable(False)
    a_ms, a_n = vc.profile_read("kmeans_assign")
    u_ms, u_n = vc.profile_read("kmeans_update")
    f_ms, f_n = vc.profile_read("kmeans_finalize")
    s_ms, s_n = vc.profile_read("kmeans_sums")
    a_flops = 2.0 * n_loc * KM_K * KM_D
    a_ach = a_flops / (a_ms / max(a_n, 1) / 1e3) / 1e12
    out = {
        "metric": f"k-means iterations/s ({w['name']})",
        "value": res.iterations / loop_s, "unit": "iterations/s", "higher_is_better": True,
        "n_gpus": world, "iterations": res.iterations, "inertia": res.inertia, "loop_seconds": loop_s,
        "fit_call_seconds": km_s, "fit_call_iterations_per_s": res.iterations / km_s,
        "config": {"workload": w["name"], "n": KMN, "dim": KM_D, "K": KM_K, "sigma": w["sigma"],
                   "init": "the first K points", "tol": 0.0,
                   "parallelism": f"row-sharded x{world} + NCCL all-reduce of the sums"},
        "timing": "CUDA events around the Lloyd loop inside vrs_kmeans_fit_rank (points resident "
                  "in HBM; the loop includes each iteration's convergence readback; upload, operand "
                  "prep and initial centroids excluded), max over ranks; "
                  "fit_call_* times the whole call on the host",
        "assign_roofline": {"bound": "tensor", "achieved": a_ach, "peak": ctx.peak_burst,
                            "unit": "TFLOP/s", "frac": a_ach / ctx.peak_burst,
                            "peak_source": f"{ctx.pk_kind} bf16 dense, burst",
                            "frac_of_sustained": a_ach / ctx.peak_sus,
                            "flops_per_launch": a_flops,
                            "per_launch_ms": a_ms / max(a_n, 1), "launches": a_n},
        "update_ms_per_launch": u_ms / max(u_n, 1),
        "finalize_ms_per_launch": f_ms / max(f_n, 1),
        "sums_ms_per_launch": s_ms / max(s_n, 1),
        "clocks": clk.summary()}

    if sustained:
        # Whole fits back to back for at least one second of Lloyd loop (its
        # count from the median loop time of three fits, agreed by all ranks);
        # the line's value is this region's rate, the single fit above is
        # kept as `single_fit_*` (one 20-iteration loop is only ~16 ms, so
        # one host hiccup moves it).
        probe = []
        for _ in range(3):
            vc.profile_reset()
            vc.profile_enable(2)
            fit(w["iters"])
            vc.profile_enable(False)
            probe.append(vc.profile_read("kmeans_loop")[0] / 1e3)
        vc.profile_reset()
        vc.profile_enable(2)
        n_fit = max(1, int(np.ceil(1.2 / max(float(np.median(probe)), 1e-4))))
        n_fit = int(max_over_ranks(float(n_fit)))
        iters = 0
        with ClockSampler(ctx.local) as clk_s:
            barrier()
            for _ in range(n_fit):
                iters += fit(w["iters"]).iterations
            barrier()
        vc.profile_enable(False)
        ls = max_over_ranks(vc.profile_read("kmeans_loop")[0] / 1e3)
        out["sustained"] = {"fits": n_fit, "iterations": iters, "loop_seconds": ls, "value": iters / ls,
                            "clocks": clk_s.summary()}
        out["single_fit_value"] = out["value"]
        out["value"] = iters / ls
        out["timing"] = ("CUDA events around every Lloyd loop of back-to-back vrs_kmeans_fit_rank calls, at "
                         "least one second of loops (points resident in HBM; each loop includes its "
                         "iterations' convergence readbacks; upload, operand prep and initial centroids "
                         "excluded), max over ranks; single_fit_value is one fit; fit_call_* times one "
                         "whole call on the host")

    if e2e:
        # Through the C ABI with host buffers: every rank's points are read
        # from host memory and the centroids and its assignments come back to
        # host memory inside the timed call (operand prep included).
        x_host = xs[:n_loc].cpu().numpy()
        vc.kmeans_fit_rank(ctx.comm, x_host, KMN, KM_D, KM_K, init_h, 1, 0.0, M)
        with ClockSampler(ctx.local) as clk_e:
            barrier()
            t0 = time.perf_counter()
            r_e = vc.kmeans_fit_rank(ctx.comm, x_host, KMN, KM_D, KM_K, init_h, w["iters"], 0.0, M)
            e_s = max_over_ranks(time.perf_counter() - t0)
            barrier()
        out["e2e"] = {"value": r_e.iterations / e_s, "unit": "iterations/s", "seconds": e_s,
                      "h2d_bytes_per_step": KMN * KM_D * 4 + world * KM_K * KM_D * 4,
                      "d2h_bytes_per_step": world * KM_K * KM_D * 4 + KMN * 4,
                      "how": "one vrs_kmeans_fit_rank per rank on host buffers (points, init in; centroids "
                             "and assignments out), host clock around the call, max over ranks",
                      "clocks": clk_e.summary()}
        del x_host

    # ------------------------------------- parity (every N) and CPU baseline
    if parity_iters > 0:
        r_p = fit(parity_iters)
        a_local = torch.from_numpy(r_p.assignments.astype(np.int32)).to(dev)
        if parity_sample:
            a_all = a_local[:parity_sample] if rank == 0 else None  # rank 0's first rows are global rows
        else:
            a_all = ctx.gather_rows(a_local)
        if rank == 0:
            orc = oracle_mod()
            cores = host_cores()
            nx = parity_sample or KMN
            full = torch.empty((nx, KM_D), dtype=torch.float32, device=dev)
            vc.gen_rows_device(vc.GEN_MIXTURE, km_seed, w["stream_x"], 0, nx, KM_D, full.data_ptr(),
                               cent.data_ptr(), KM_K, w["sigma"])
            torch.cuda.synchronize()
            x_h = full.cpu().numpy()
            del full
            g_assign = a_all.cpu().numpy()
            t0 = time.perf_counter()
            if parity_sample:
                o_assign, _, _, _ = orc.kmeans_local(x_h, init_h, L2, nthreads=cores)
                dt = time.perf_counter() - t0
                out["parity"] = {"iterations": 1, "points": nx,
                                 "assign_equal_frac": float((g_assign[:nx] == o_assign).mean()),
                                 "n_gpus": world,
                                 "how": "assignments of the first Lloyd step (against the initial "
                                        f"centroids) for the first {nx} points vs the oracle"}
            else:
                c_o, o_assign, it_o, in_o = orc.kmeans_fit(x_h, KM_K, init_h, parity_iters, 0.0, L2,
                                                           nthreads=cores)
                dt = time.perf_counter() - t0
                out["parity"] = {
                    "iterations": int(it_o), "points": nx, "n_gpus": world,
                    "assign_equal_frac": float((g_assign == o_assign).mean()),
                    "inertia_gpu": r_p.inertia, "inertia_oracle": in_o,
                    "inertia_rel_err": abs(r_p.inertia - in_o) / max(abs(in_o), 1e-30),
                    "centroid_max_abs_err": float(np.abs(r_p.centroids - c_o).max()),
                    "how": f"same init, {parity_iters} Lloyd iterations on all points, oracle fit_cpu restatement"}
                if cpu_leg and world == 1:
                    out["cpu_baseline"] = {
                        "value": it_o / dt, "unit": "iterations/s", "cores": cores, "kind": "port",
                        "sample": f"{it_o} of the {w['iters']} Lloyd iterations on all {nx} points "
                                  f"(AVX-512 restatement of fit_cpu, {cores} threads)",
                        "seconds": dt}
        del a_local, a_all
    del xs, cent, init
    torch.cuda.empty_cache()
    barrier()
    return out


def ivf_bench(args, vc, torch, dev, peak_tc):  # peak_tc: bf16 burst
    """IVF coarse quantiser on the C5b shape (the quantiser C5b trains):
    nlist = 16,384 centroids x 96, squared L2. Probes 10,000 queries at
    nprobe = 32 (KMeans::find_top_centroids per query in IvfPqIndex::search,
    crates/vector-index/src/ivf/mod.rs:277-284) and assigns 1,000,000 base
    rows (find_nearest_centroid per row in IvfPqIndex::build, mod.rs:119-125),
    each as one call of vrs_ivf_find_top_centroids / vrs_ivf_assign on host
    buffers (host->device copies, search, device->host copies all timed)."""
    K, D, NQ, P, NA, SIGMA = 16_384, 96, 10_000, 32, 1_000_000, 0.05
    seed = vc.config_seed(4)
    cent = torch.empty((K, D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_NORMAL, seed, 5, 0, K, D, cent.data_ptr())
    q = torch.empty((NQ, D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_MIXTURE, seed, 7, 0, NQ, D, q.data_ptr(), cent.data_ptr(), K, SIGMA)
    xa = torch.empty((NA, D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_MIXTURE, seed, 6, 0, NA, D, xa.data_ptr(), cent.data_ptr(), K, SIGMA)
    cent_h, q_h, xa_h = cent.cpu().numpy(), q.cpu().numpy(), xa.cpu().numpy()
    del cent, q, xa
    torch.cuda.empty_cache()
    cq = vc.CoarseQuantizer(cent_h, D, vc.DistanceMetric.L2Squared)
    for _ in range(max(args.warmup, 3)):
        cq.find_top_centroids(q_h, P)
    cq.assign(xa_h[:NQ])
    steps = max(args.steps, 1)
    with ClockSampler(dev.index or 0) as clk:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            sg, ig = cq.find_top_centroids(q_h, P)
        probe_s = (time.perf_counter() - t0) / steps
        t0 = time.perf_counter()
        ia, sa = cq.assign(xa_h)
        assign_s = time.perf_counter() - t0
    # Device-side breakdown of one probe call (every stage bracketed by events).
    vc.profile_reset()
    vc.profile_enable(True)
    cq.find_top_centroids(q_h, P)
    vc.profile_enable(False)
    stages = {}
    for nm in ("knn_prep", "knn_pivot", "knn_scan", "knn_select", "knn_fallback"):
        ms, n = vc.profile_read(nm)
        stages[nm] = {"ms": ms, "launches": n}
    scan_ms = stages["knn_scan"]["ms"]
    flops = 2.0 * NQ * K * D
    ach = flops / (scan_ms / 1e3) / 1e12 if scan_ms > 0 else None
    # Parity sample and CPU baseline from the oracle (the restated reference loop).
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    S = 300
    so, io = oracle.find_top_centroids_batch(q_h[:S], cent_h, P, 0)
    cores = os.cpu_count() or 1
    t0 = time.perf_counter()
    oracle.knn_search(cent_h, q_h[:S], P, 0, nthreads=cores)
    cpu_s = time.perf_counter() - t0
    cq.close()
    return {
        "metric": "IVF coarse probe queries/s (nlist 16384 x 96, squared L2, nprobe 32)",
        "value": NQ / probe_s, "unit": "queries/s", "higher_is_better": True, "n_gpus": 1,
        "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": probe_s * 1e3,
        "dtype": "f32 (fp16 tensor-core scan with exact f32 re-rank)", "data": "synthetic",
        "config": {"workload": "IVF quantiser of C5b: 16,384 x 96 centroids N(0,1), queries and "
                               "base rows a Gaussian mixture around them (sigma 0.05)",
                   "nlist": K, "dim": D, "queries_per_step": NQ, "nprobe": P, "assign_rows": NA,
                   "l2": "no flush: the 6.3 MB of centroids stay L2-resident across calls, as "
                         "in serving; queries come from host memory in every call"},
        "timing": "host clock around the synchronous C-ABI call on host buffers (copies included)",
        "e2e": {"value": NQ / probe_s, "unit": "queries/s", "h2d_bytes_per_step": NQ * D * 4,
                "d2h_bytes_per_step": NQ * P * 8},
        "assign": {"value": NA / assign_s, "unit": "rows/s", "seconds": assign_s,
                   "h2d_bytes": NA * D * 4, "d2h_bytes": NA * 12},
        "stages": stages,
        "roofline": {"bound": "tensor", "achieved": ach, "peak": peak_tc, "unit": "TFLOP/s",
                     "frac": ach / peak_tc if ach else None, "traffic": None,
                     "note": "knn_scan over one probe call, algorithmic 2*nq*nlist*dim FLOP"},
        "parity": {"queries": S, "ids_equal_frac": float((ig[:S] == io).mean()),
                   "score_bit_equal_frac": float((sg[:S].view(np.uint32) == so.view(np.uint32)).mean())},
        "cpu_baseline": {"value": S / cpu_s, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": f"{S} queries, oracle batch kNN at k = nprobe over all centroids"},
        "clocks": clk.summary(),
        "gpu_launches": sum(v["launches"] for v in stages.values()),
    }


def ivfpq_bench(args, vc, torch, dev, pk, pk_kind):
    """IVF-PQ ADC search (IvfPqIndex::search_with_nprobe,
    crates/vector-index/src/ivf/mod.rs:265-345) on an index of the C5b shape:
    nlist = 16,384 coarse centroids over d = 96 (the quantiser C5b trains),
    10,000,000 encoded rows with M = 16 sub-spaces of 256 sub-centroids;
    10,000 queries per step around the centroids, nprobe = 32, k = 100. One
    step = one vrs_ivfpq_search on host buffers (coarse probe, ADC tables,
    scores, heaps, copies). Codes are drawn uniformly and list sizes from a
    uniform multinomial (the ADC work does not depend on code values)."""
    K, D, M, KS, N, NQ, P, KK = 16_384, 96, 16, 256, 10_000_000, 10_000, 32, 100
    seed = vc.config_seed(4)
    rng = np.random.default_rng(seed & 0xFFFFFFFF)
    cent = torch.empty((K, D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_NORMAL, seed, 5, 0, K, D, cent.data_ptr())
    q = torch.empty((NQ, D), dtype=torch.float32, device=dev)
    vc.gen_rows_device(vc.GEN_MIXTURE, seed, 7, 0, NQ, D, q.data_ptr(), cent.data_ptr(), K, 0.05)
    cent_h, q_h = cent.cpu().numpy(), q.cpu().numpy()
    del cent, q
    cb = (0.05 * rng.standard_normal(M * KS * (D // M))).astype(np.float32)
    sizes = rng.multinomial(N, np.full(K, 1.0 / K))
    off = np.zeros(K + 1, np.int64)
    off[1:] = np.cumsum(sizes)
    ids = rng.permutation(N).astype(np.uint32)
    codes = rng.integers(0, KS, (N, M), dtype=np.uint8)
    lists = [(ids[off[c]:off[c + 1]], codes[off[c]:off[c + 1]]) for c in range(K)]
    ids_flat, codes_flat = ids, codes  # lists back to back already
    idx = vc.IvfPqIndex(cent_h, D, cb, M, KS, lists, vc.DistanceMetric.L2Squared)
    for _ in range(max(args.warmup, 3)):
        idx.search_batch(q_h, KK, P)
    steps = max(args.steps, 1)
    with ClockSampler(dev.index or 0) as clk:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            gd, gi, gc = idx.search_batch(q_h, KK, P)
        step_s = (time.perf_counter() - t0) / steps
    vc.profile_reset()
    vc.profile_enable(True)
    idx.search_batch(q_h, KK, P)
    vc.profile_enable(False)
    adc_ms, adc_n = vc.profile_read("ivfpq_adc")
    stages = {nm: dict(zip(("ms", "launches"), vc.profile_read(nm)))
              for nm in ("knn_prep", "knn_pivot", "knn_scan", "knn_select", "ivfpq_adc")}
    launches = sum(v["launches"] for v in stages.values())
    idx.close()
    # Parity sample and CPU baseline: the oracle's C restatement of the
    # reference search, one query per call, calls spread over host threads.
    orc = oracle_mod()
    import ivfpq
    from concurrent.futures import ThreadPoolExecutor
    S = 64
    cores = host_cores()

    def one(i):
        return ivfpq.ivf_pq_search_c_flat(q_h[i], KK, P, cent_h, off, ids_flat, codes_flat, cb, M, KS, L2)

    t0 = time.perf_counter()
    with ThreadPoolExecutor(cores) as ex:
        ref = list(ex.map(one, range(S)))
    cpu_s = time.perf_counter() - t0
    ids_eq = np.mean([np.array_equal(gi[i, :gc[i]], ref[i][1]) for i in range(S)])
    dist_eq = np.mean([np.array_equal(gd[i, :gc[i]].view(np.uint32), ref[i][0].view(np.uint32)) for i in range(S)])
    cand = float(np.mean([sizes[c] for c in range(K)])) * P
    bytes_q = cand * (M + 4)  # codes + ids of the probed lists
    ach = bytes_q * NQ / (adc_ms / max(adc_n, 1) / 1e3) / 1e9
    del orc
    return {
        "metric": "IVF-PQ ADC search queries/s (nlist 16384, d 96, M 16 x 256, 10M rows, nprobe 32, k 100)",
        "value": NQ / step_s, "unit": "queries/s", "higher_is_better": True, "n_gpus": 1,
        "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": step_s * 1e3,
        "dtype": "f32 tables and sums (the reference's arithmetic)", "data": "synthetic",
        "config": {"workload": "IVF-PQ index of the C5b shape: coarse centroids N(0,1), queries a mixture "
                               "around them (sigma 0.05), codebooks N(0, 0.05^2), uniform codes, list sizes "
                               "multinomial(10M, uniform)",
                   "nlist": K, "dim": D, "num_subvectors": M, "sub_clusters": KS, "rows": N,
                   "queries_per_step": NQ, "nprobe": P, "k": KK,
                   "l2": "codes + ids 200 MB, larger than L2; queries from host memory every call"},
        "timing": "host clock around the synchronous vrs_ivfpq_search on host buffers (probe, ADC, copies)",
        "e2e": {"value": NQ / step_s, "unit": "queries/s", "h2d_bytes_per_step": NQ * D * 4 * 2 + NQ * P * 4,
                "d2h_bytes_per_step": NQ * (KK * 8 + 4) + NQ * P * 12},
        "stages": stages,
        "roofline": {"bound": "hbm", "kernel": "ivfpq_adc", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": ach / pk["hbm_gbs"], "peak_source": f"{pk_kind} HBM copy",
                     "bytes_per_query": bytes_q, "traffic": None,
                     "note": "algorithmic bytes = codes + ids of the probed lists per query; lists shared by "
                             "queries are re-read from L2, so the kernel is bound by its table builds and "
                             "shared-memory lookups rather than HBM"},
        "parity": {"queries": S, "ids_equal_frac": float(ids_eq), "dist_bit_equal_frac": float(dist_eq)},
        "cpu_baseline": {"value": S / cpu_s, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": f"{S} queries, oracle C restatement of search_with_nprobe, one query per call "
                                   f"on {cores} threads"},
        "clocks": clk.summary(),
        "gpu_launches": launches,
    }


def storage_bench(args, vc, torch, dev, pk):
    """Loading a base from a VECRSTOR file (crates/vector-index/src/storage/mmap.rs)
    into a one-GPU engine: vrs_knn_create_from_file (validate, map, upload
    from the mapping) against vrs_knn_create from the same rows already in
    host memory. The file is written first, so it is read from the page cache."""
    import tempfile
    N, D = args.n_base or 5_000_000, 96
    rows = host_gen(vc, vc.GEN_NORMAL, vc.config_seed(4), 0, N, D)
    fd, path = tempfile.mkstemp(suffix=".vecrstor", dir=os.environ.get("TMPDIR", "/tmp"))
    os.close(fd)
    try:
        vc.MmapStorage.create_from_flat(path, D, rows)
        M = vc.DistanceMetric.L2Squared
        vc.DistributedKnnEngine.from_file(path, 1, vc.GpuShardMode.Sharded, M).close()  # warm
        t_file, t_mem = [], []
        for _ in range(max(args.steps, 1)):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            e = vc.DistributedKnnEngine.from_file(path, 1, vc.GpuShardMode.Sharded, M)
            t_file.append(time.perf_counter() - t0)
            e.close()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            e = vc.DistributedKnnEngine.try_new(rows, D, 1, vc.GpuShardMode.Sharded, M)
            t_mem.append(time.perf_counter() - t0)
            e.close()
    finally:
        os.unlink(path)
    gb = N * D * 4 / 1e9
    tf, tm = float(np.median(t_file)), float(np.median(t_mem))
    return {"metric": "VECRSTOR file -> GPU engine load GB/s (rows of f32)", "value": gb / tf,
            "unit": "GB/s", "higher_is_better": True, "n_gpus": 1, "steps": len(t_file),
            "seconds_file": tf, "seconds_from_host_array": tm, "gb": gb,
            "from_host_array_gbs": gb / tm, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{N} x {D} N(0,1) rows in one VECRSTOR file (page cache)",
                       "metric": "squared L2 (norms computed at upload)"},
            "timing": "host clock around the synchronous create call, median of steps"}


if __name__ == "__main__":
    sys.exit(main())
