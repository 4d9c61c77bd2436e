"""ctypes wrapper for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_build/liboracle.so`` (built by ``oracle/Makefile``). Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module; the product never does.

The functions restate VectorRS's CPU paths (see ``vrs_oracle.c``):
``knn_search`` = ``CudaKnnEngine::search_batch_cpu``
(crates/vector-cuda/src/knn.rs:312-377), ``kmeans_fit`` =
``CudaKMeansEngine::fit_cpu`` (crates/vector-cuda/src/kmeans.rs:240-357),
``topk_reduce`` = ``CollectiveOps::top_k_reduce``
(crates/vector-cuda/src/ddp/collective.rs:115-159), ``distance`` = the
AVX-512 pair kernels of crates/vector-simd/src/avx512.rs.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_distance.restype = ctypes.c_float
        L.orc_distance.argtypes = [ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_rank_key.restype = ctypes.c_float
        L.orc_rank_key.argtypes = [ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_has_avx512.restype = ctypes.c_int
        L.orc_knn_search.restype = ctypes.c_int
        L.orc_knn_search.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_int64,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     _f32p, _u32p, ctypes.POINTER(ctypes.c_int)]
        L.orc_topk_reduce.restype = ctypes.c_int
        L.orc_topk_reduce.argtypes = [_f32p, _u32p, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      _f32p, _u32p]
        L.orc_kmeans_fit.restype = ctypes.c_int
        L.orc_kmeans_fit.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p,
                                     ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, _f32p, ctypes.c_void_p,
                                     ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)]
        L.orc_knn_search_rows.restype = ctypes.c_int
        L.orc_knn_search_rows.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_uint32, _f32p, _u32p, ctypes.POINTER(ctypes.c_int)]
        L.orc_gen_rows.restype = ctypes.c_int
        L.orc_gen_rows.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int64,
                                   ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_void_p, ctypes.c_uint32,
                                   ctypes.c_double, ctypes.c_int]
        L.orc_kmeans_local.restype = None
        L.orc_kmeans_local.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.POINTER(ctypes.c_double)]
        L.orc_kmeans_update.restype = ctypes.c_float
        L.orc_kmeans_update.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                        _f32p]
        _lib = L
    return _lib


def has_avx512() -> bool:
    return bool(lib().orc_has_avx512())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def distance(metric: int, a, b, use_simd: int = -1) -> float:
    a, b = _f32(a).ravel(), _f32(b).ravel()
    assert a.size == b.size
    return float(lib().orc_distance(int(metric), a, b, a.size, use_simd))


def rank_key(metric: int, a, b, use_simd: int = -1) -> float:
    a, b = _f32(a).ravel(), _f32(b).ravel()
    return float(lib().orc_rank_key(int(metric), a, b, a.size, use_simd))


def knn_search(base, queries, k: int, metric: int, nthreads: int | None = None, use_simd: int = -1):
    """Returns (dist[nq,k'], ids[nq,k']) best-first, k' = min(k, n)."""
    base, queries = _f32(base), _f32(queries)
    n, d = base.shape
    nq = queries.shape[0]
    kk = max(0, min(k, n))
    out_d = np.zeros((nq, max(kk, 1)), np.float32)
    out_i = np.zeros((nq, max(kk, 1)), np.uint32)
    ok = ctypes.c_int(0)
    lib().orc_knn_search(base, n, d, queries, nq, int(k), int(metric),
                         int(nthreads or os.cpu_count() or 1), use_simd, out_d, out_i, ctypes.byref(ok))
    return out_d[:, :ok.value], out_i[:, :ok.value]


def knn_search_rows(base, queries, k: int, metric: int, nthreads: int | None = None, use_simd: int = -1,
                    id_offset: int = 0):
    """knn_search for a few queries over many rows (threads split the rows;
    identical results). Ids are row index + id_offset."""
    base, queries = _f32(base), _f32(queries)
    n, d = base.shape
    nq = queries.shape[0]
    kk = max(0, min(k, n))
    out_d = np.zeros((nq, max(kk, 1)), np.float32)
    out_i = np.zeros((nq, max(kk, 1)), np.uint32)
    ok = ctypes.c_int(0)
    lib().orc_knn_search_rows(base, n, d, queries, nq, int(k), int(metric), int(nthreads or os.cpu_count() or 1),
                              use_simd, int(id_offset), out_d, out_i, ctypes.byref(ok))
    return out_d[:, :ok.value], out_i[:, :ok.value]


# Generator kinds (the product's VRS_GEN_* values).
GEN_NORMAL, GEN_NORMAL_UNIT, GEN_UNIFORM, GEN_UNIFORM_SUM1, GEN_MIXTURE = 0, 1, 2, 3, 4


def gen_rows(kind: int, seed: int, stream: int, row0: int, rows: int, d: int, centres=None, K: int = 0,
             sigma: float = 0.0, nthreads: int | None = None) -> np.ndarray:
    """Rows [row0, row0 + rows) of a seeded synthetic matrix (orc_gen.c), the
    same bits the product's generator gives, without loading libvrs."""
    out = np.empty((rows, d), np.float32)
    cp = None
    if centres is not None:
        centres = _f32(centres)
        cp = centres.ctypes.data
    if rows > 0:
        st = lib().orc_gen_rows(int(kind), int(seed), int(stream), int(row0), int(rows), int(d), out, cp,
                                int(K), float(sigma), int(nthreads or os.cpu_count() or 1))
        if st != 0:
            raise ValueError("orc_gen_rows: bad arguments")
    return out


def config_seed(index: int) -> int:
    """Seed of benchmark config `index`: "VRS_B001" as a 64-bit integer + index."""
    return 0x5652535F42303031 + int(index)


def topk_reduce(lists, k: int, metric: int):
    """lists: sequence of (dists, ids) per rank, in rank order."""
    lens = np.array([len(d) for d, _ in lists] or [0], np.int32)
    dists = _f32(np.concatenate([np.asarray(d, np.float32) for d, _ in lists]) if lists else np.zeros(1))
    ids = np.ascontiguousarray(np.concatenate([np.asarray(i, np.uint32) for _, i in lists]) if lists
                               else np.zeros(1, np.uint32), dtype=np.uint32)
    out_d = np.zeros(max(k, 1), np.float32)
    out_i = np.zeros(max(k, 1), np.uint32)
    m = lib().orc_topk_reduce(dists, ids, lens, len(lists), int(k), int(metric), out_d, out_i)
    return out_d[:m], out_i[:m]


def kmeans_fit(x, k: int, init, max_iters: int, tol: float, metric: int,
               nthreads: int | None = None, use_simd: int = -1):
    """Returns (centroids[k',d], assign[n], iterations, inertia(f64))."""
    x = _f32(x)
    n, d = x.shape
    kk = max(0, min(k, n))
    init = _f32(init).reshape(-1)
    cent = np.zeros(max(kk * d, 1), np.float32)
    assign = np.zeros(max(n, 1), np.int32)
    it = ctypes.c_int(0)
    inertia = ctypes.c_double(0.0)
    kk = lib().orc_kmeans_fit(x, n, d, int(k), init, int(max_iters), float(tol), int(metric),
                              int(nthreads or os.cpu_count() or 1), use_simd, cent,
                              assign.ctypes.data, ctypes.byref(it), ctypes.byref(inertia))
    return cent[:kk * d].reshape(kk, d), assign[:n], it.value, inertia.value


def kmeans_local(x, centroids, metric: int, nthreads: int | None = None, use_simd: int = -1):
    """One rank's share of a Lloyd iteration on its rows x.
    Returns (assign[n], sums[k,d] f64, counts[k] i64, inertia f64)."""
    x = _f32(x).reshape(-1, np.asarray(centroids).shape[1])
    cent = _f32(centroids)
    n, d = x.shape
    kk = cent.shape[0]
    assign = np.zeros(max(n, 1), np.int32)
    sums = np.zeros((kk, d), np.float64)
    counts = np.zeros(kk, np.int64)
    inertia = ctypes.c_double(0.0)
    lib().orc_kmeans_local(x, n, d, kk, cent, int(metric), int(nthreads or os.cpu_count() or 1),
                           use_simd, assign.ctypes.data, sums.ctypes.data, counts.ctypes.data,
                           ctypes.byref(inertia))
    return assign[:n], sums, counts, inertia.value


def kmeans_update(sums, counts, centroids):
    """In-place centroid update from global sums/counts; returns the largest
    squared shift."""
    sums = np.ascontiguousarray(sums, np.float64)
    counts = np.ascontiguousarray(counts, np.int64)
    assert centroids.dtype == np.float32 and centroids.flags.c_contiguous
    kk, d = centroids.shape
    return float(lib().orc_kmeans_update(sums.ctypes.data, counts.ctypes.data, kk, d, centroids))


# ---------------------------------------------------------------------------
# IVF coarse quantiser: KMeans::find_nearest_centroid / find_top_centroids
# (crates/vector-index/src/ivf/kmeans.rs:264-356), pair values from the same
# AVX-512 restatement as everything above.
# ---------------------------------------------------------------------------

HIGHER_IS_BETTER = (1, 2)  # DotProduct, CosineSimilarity (crates/vector-index/src/lib.rs:89-94)


def find_nearest_centroid(vector, centroids, metric: int):
    """kmeans.rs:264-309, literally: start from (0, +inf) (-inf for
    similarities), walk the centroids in order, replace on a strict
    improvement only."""
    centroids = _f32(centroids)
    hib = metric in HIGHER_IS_BETTER
    best_idx, best = 0, (-np.inf if hib else np.inf)
    for c in range(centroids.shape[0]):
        v = distance(metric, vector, centroids[c])
        if (v > best) if hib else (v < best):
            best_idx, best = c, v
    return best_idx, np.float32(best)


def find_top_centroids(query, centroids, nprobe: int, metric: int):
    """kmeans.rs:312-356, literally: score every centroid in index order,
    stable sort by score (descending for similarities), keep min(nprobe, K)."""
    centroids = _f32(centroids)
    target = min(nprobe, centroids.shape[0])
    if target == 0:
        return []
    scored = [(c, distance(metric, query, centroids[c])) for c in range(centroids.shape[0])]
    scored.sort(key=lambda t: t[1], reverse=metric in HIGHER_IS_BETTER)  # stable both ways
    return [(c, np.float32(v)) for c, v in scored[:target]]


def find_top_centroids_batch(queries, centroids, nprobe: int, metric: int,
                             nthreads: int | None = None):
    """The same result for many queries at once: every centroid scored by the
    batch kNN restatement (k = K, all reported values), then each row
    ordered by (value, index) -- the stable sort of kmeans.rs:345-350 -- and
    cut to min(nprobe, K). Returns (scores[nq, P] f32, indices[nq, P] int64)."""
    centroids, queries = _f32(centroids), _f32(queries)
    K = centroids.shape[0]
    nq = queries.shape[0]
    p = min(nprobe, K)
    if p == 0 or nq == 0:
        return np.zeros((nq, 0), np.float32), np.zeros((nq, 0), np.int64)
    dist, ids = knn_search(centroids, queries, K, metric, nthreads)
    sign = -1.0 if metric in HIGHER_IS_BETTER else 1.0
    out_s = np.empty((nq, p), np.float32)
    out_i = np.empty((nq, p), np.int64)
    for r in range(nq):
        order = np.lexsort((ids[r].astype(np.int64), sign * dist[r].astype(np.float64)))[:p]
        out_s[r] = dist[r][order]
        out_i[r] = ids[r][order]
    return out_s, out_i
