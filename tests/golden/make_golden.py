#!/usr/bin/env python
"""Writes the golden fixtures of this directory.

    python tests/golden/make_golden.py

Inputs are seeded Philox4x32-10 rows from libvrs's host generator
(vrs_gen_rows_host; bit-identical to the device generator), so a fixture
stores only the seed and shapes plus the expected outputs. Outputs are the
CPU oracle's (the AVX-512 restatement of the reference's search_batch_cpu,
crates/vector-cuda/src/knn.rs:181-216, and of the CPU Lloyd loop,
crates/vector-cuda/src/kmeans.rs:99-160), computed with the SIMD path the
reference takes on an AVX-512 host.

knn_golden.npz: per metric 0..9, a 3000 x 37 base, 8 queries, k = 16
  (dist bits + ids), plus a 4096 x 128 cosine case (k = 100).
kmeans_golden.npz: 4000 x 16 Gaussian mixture, K = 8, 15 Lloyd iterations
  for L2 and cosine (centroid bits, assignments, iterations, inertia).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vector-rs_b200", "python"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

L2, DOT, COS, L1, MINK, CHEB, HAM, MAHA, JAC, HELL = range(10)

KNN_N, KNN_D, KNN_Q, KNN_K = 3000, 37, 8, 16
BIG_N, BIG_D, BIG_Q, BIG_K = 4096, 128, 16, 100
KM_N, KM_D, KM_K, KM_ITERS, KM_SIGMA = 4000, 16, 8, 15, 0.3


def knn_kind(vc, metric):
    if metric == HELL:
        return vc.GEN_UNIFORM_SUM1
    if metric in (L1, CHEB, JAC):
        return vc.GEN_UNIFORM
    if metric == COS:
        return vc.GEN_NORMAL_UNIT
    return vc.GEN_NORMAL


def knn_inputs(vc, metric):
    """(base, queries) of the per-metric case; Hamming rows are quantised to
    halves so its distances tie often."""
    s = vc.config_seed(500 + metric)
    kind = knn_kind(vc, metric)
    base = vc.gen_rows_host(kind, s, 0, 0, KNN_N, KNN_D)
    qs = vc.gen_rows_host(kind, s, 1, 0, KNN_Q, KNN_D)
    if metric == HAM:
        base, qs = np.round(base * 2) / 2, np.round(qs * 2) / 2
    return np.ascontiguousarray(base, np.float32), np.ascontiguousarray(qs, np.float32)


def big_inputs(vc):
    s = vc.config_seed(520)
    return (vc.gen_rows_host(vc.GEN_NORMAL_UNIT, s, 0, 0, BIG_N, BIG_D),
            vc.gen_rows_host(vc.GEN_NORMAL_UNIT, s, 1, 0, BIG_Q, BIG_D))


def kmeans_inputs(vc):
    """(points, initial centroids): a mixture around K seeded centres; the
    initial centroids are K further draws of the same mixture."""
    s = vc.config_seed(530)
    cent = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, KM_K, KM_D)
    x = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 0, KM_N, KM_D, cent, KM_K, KM_SIGMA)
    init = vc.gen_rows_host(vc.GEN_MIXTURE, s, 3, 0, KM_K, KM_D, cent, KM_K, KM_SIGMA)
    return x, init


def main():
    import oracle
    import vector_cuda as vc
    oracle.build()
    if not oracle.has_avx512():
        raise SystemExit("fixtures follow the reference's AVX-512 path: run on an AVX-512 host")
    out = {}
    for m in range(10):
        base, qs = knn_inputs(vc, m)
        d, i = oracle.knn_search(base, qs, KNN_K, m, use_simd=1)
        out[f"m{m}_dist_bits"] = d.view(np.uint32)
        out[f"m{m}_ids"] = i
        out[f"m{m}_base_sum"] = np.float64(base.astype(np.float64).sum())
    base, qs = big_inputs(vc)
    d, i = oracle.knn_search(base, qs, BIG_K, COS, use_simd=1)
    out["big_dist_bits"] = d.view(np.uint32)
    out["big_ids"] = i
    np.savez_compressed(os.path.join(HERE, "knn_golden.npz"), **out)

    x, init = kmeans_inputs(vc)
    km = {}
    for m in (L2, COS):
        c, a, it, inertia = oracle.kmeans_fit(x, KM_K, init, KM_ITERS, 0.0, m, use_simd=1)
        km[f"m{m}_centroid_bits"] = c.view(np.uint32)
        km[f"m{m}_assign"] = a
        km[f"m{m}_iters"] = np.int32(it)
        km[f"m{m}_inertia"] = np.float64(inertia)
    km["x_sum"] = np.float64(x.astype(np.float64).sum())
    np.savez_compressed(os.path.join(HERE, "kmeans_golden.npz"), **km)
    print("wrote", sorted(out)[:3], "...", sorted(km))


if __name__ == "__main__":
    main()
