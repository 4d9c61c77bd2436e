/*
 * caller.c -- a plain C program that uses libvrs only through include/vrs.h,
 * the way the reference's Rust crate would bind it (crates/vector-cuda/src/
 * lib.rs:20-26 re-exports the engines this ABI stands in for).
 *
 *   caller            no GPU needed: device count, argument and device errors
 *   caller gpu        also: create/search/destroy and a k-means fit on GPU 0
 *
 * Prints one line per check and exits non-zero on the first failure.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "vrs.h"

#define CHECK(cond, ...)                                  \
  do {                                                    \
    if (!(cond)) {                                        \
      fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      fprintf(stderr, __VA_ARGS__);                       \
      fprintf(stderr, " (last error: %s)\n", vrs_last_error()); \
      return 1;                                           \
    }                                                     \
  } while (0)

/* xorshift64* -> uniform in [-1, 1) */
static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static float urand(void) {
  rng_state ^= rng_state >> 12;
  rng_state ^= rng_state << 25;
  rng_state ^= rng_state >> 27;
  uint64_t x = rng_state * 0x2545F4914F6CDD1Dull;
  return (float)((double)(x >> 40) / (double)(1ull << 24) * 2.0 - 1.0);
}

static int cpu_checks(int ndev) {
  vrs_knn* h = NULL;
  float base[8] = {0};
  int st = vrs_knn_create(base, 4, 2, ndev + 1, VRS_SHARDED, VRS_L2_SQUARED, &h);
  CHECK(st == VRS_ERR_INSUFFICIENT_DEVICES && h == NULL, "too many GPUs gave %d", st);
  CHECK(strstr(vrs_last_error(), "Insufficient") != NULL, "message names the shortage");
  st = vrs_knn_create(base, 4, 2, 1, VRS_SHARDED, 42, &h);
  CHECK(st == VRS_ERR_INVALID_CONFIG || st == VRS_ERR_INSUFFICIENT_DEVICES, "bad metric gave %d", st);
  st = vrs_knn_search(NULL, NULL, 0, 1, NULL, NULL, NULL);
  CHECK(st == VRS_ERR_INVALID_CONFIG, "null handle gave %d", st);
  int32_t k = 0, it = 0;
  double inertia = 0;
  st = vrs_kmeans_fit(base, 4, 2, 2, NULL, 5, 0.0f, VRS_L2_SQUARED, ndev + 1, base, NULL, &k, &it, &inertia);
  CHECK(st == VRS_ERR_INSUFFICIENT_DEVICES, "k-means on too many GPUs gave %d", st);
  CHECK(vrs_metric_higher_is_better(VRS_COSINE_SIMILARITY) == 1 && vrs_metric_higher_is_better(VRS_L2_SQUARED) == 0,
        "metric order flags");
  printf("ok cpu: device count %d, error statuses as CudaError\n", ndev);
  return 0;
}

static int gpu_checks(void) {
  enum { N = 2000, D = 32, Q = 16, K = 10 };
  float* base = malloc(sizeof(float) * N * D);
  float* q = malloc(sizeof(float) * Q * D);
  for (int i = 0; i < N * D; i++) base[i] = urand();
  for (int i = 0; i < Q * D; i++) q[i] = urand();
  vrs_knn* h = NULL;
  int st = vrs_knn_create(base, N, D, 1, VRS_SHARDED, VRS_L2_SQUARED, &h);
  CHECK(st == VRS_OK && h, "create gave %d", st);
  int64_t nv = 0;
  int32_t dim = 0, ng = 0, mode = -1, metric = -1;
  CHECK(vrs_knn_info(h, &nv, &dim, &ng, &mode, &metric) == VRS_OK && nv == N && dim == D && ng == 1 &&
            mode == VRS_SHARDED && metric == VRS_L2_SQUARED,
        "info");
  float dist[Q * K];
  uint32_t ids[Q * K];
  int32_t kk = 0;
  st = vrs_knn_search(h, q, Q, K, dist, ids, &kk);
  CHECK(st == VRS_OK && kk == K, "search gave %d, k' %d", st, kk);
  /* Brute force in double: the ids must match (random data, no near ties at
   * this size), the distances within 1e-4 relative. */
  for (int qi = 0; qi < Q; qi++) {
    double best[K];
    int bid[K];
    for (int j = 0; j < K; j++) best[j] = INFINITY, bid[j] = -1;
    for (int r = 0; r < N; r++) {
      double s = 0;
      for (int e = 0; e < D; e++) {
        double t = (double)q[qi * D + e] - (double)base[r * D + e];
        s += t * t;
      }
      if (s < best[K - 1]) {
        int j = K - 1;
        while (j > 0 && best[j - 1] > s) best[j] = best[j - 1], bid[j] = bid[j - 1], j--;
        best[j] = s, bid[j] = r;
      }
    }
    for (int j = 0; j < K; j++) {
      CHECK(ids[qi * K + j] == (uint32_t)bid[j], "query %d rank %d: id %u vs %d", qi, j, ids[qi * K + j], bid[j]);
      CHECK(fabs(dist[qi * K + j] - best[j]) <= 1e-4 * fmax(1.0, best[j]), "query %d rank %d distance", qi, j);
    }
  }
  vrs_knn_destroy(h);
  printf("ok gpu: vrs_knn_create/search/destroy, %d queries x top-%d equal to brute force\n", Q, K);

  /* k-means: four far-apart blobs, init = the first point of each blob. */
  enum { KN = 4000, KD = 8, KC = 4 };
  float* x = malloc(sizeof(float) * KN * KD);
  float init[KC * KD];
  double mean[KC][KD];
  memset(mean, 0, sizeof(mean));
  for (int i = 0; i < KN; i++) {
    int c = i % KC;
    for (int e = 0; e < KD; e++) {
      x[i * KD + e] = (float)(100.0 * c * (e == c ? 1 : 0)) + 0.5f * urand();
      mean[c][e] += x[i * KD + e];
    }
  }
  for (int c = 0; c < KC; c++) memcpy(init + c * KD, x + c * KD, sizeof(float) * KD);
  float cent[KC * KD];
  int32_t assign[KN], k_out = 0, iters = 0;
  double inertia = 0;
  st = vrs_kmeans_fit(x, KN, KD, KC, init, 20, 0.0f, VRS_L2_SQUARED, 1, cent, assign, &k_out, &iters, &inertia);
  CHECK(st == VRS_OK && k_out == KC && iters >= 1 && iters <= 20, "kmeans gave %d (k %d, iters %d)", st, k_out, iters);
  for (int i = 0; i < KN; i++) CHECK(assign[i] == i % KC, "point %d assigned to %d", i, assign[i]);
  for (int c = 0; c < KC; c++)
    for (int e = 0; e < KD; e++)
      CHECK(fabs(cent[c * KD + e] - mean[c][e] / (KN / KC)) < 1e-4, "centroid %d[%d]", c, e);
  CHECK(inertia > 0 && isfinite(inertia), "inertia %g", inertia);
  printf("ok gpu: vrs_kmeans_fit %d iterations, blobs recovered, inertia %.6g\n", iters, inertia);
  free(x);
  free(base);
  free(q);
  return 0;
}

int main(int argc, char** argv) {
  int32_t ndev = -1;
  CHECK(vrs_device_count(&ndev) == VRS_OK && ndev >= 0, "device count");
  CHECK(vrs_device_count(NULL) == VRS_ERR_INVALID_CONFIG, "null out_count");
  if (cpu_checks(ndev)) return 1;
  if (argc > 1 && strcmp(argv[1], "gpu") == 0) {
    CHECK(ndev >= 1, "no GPU for the gpu checks");
    return gpu_checks();
  }
  return 0;
}
