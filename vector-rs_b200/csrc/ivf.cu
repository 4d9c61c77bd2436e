// ivf.cu -- IVF coarse-quantiser probing and assignment on the GPU.
//
// The reference's IVF index asks its coarse k-means quantiser two questions:
//   * KMeans::find_top_centroids (crates/vector-index/src/ivf/kmeans.rs:312-356):
//     the nprobe centroids nearest a query, best first, for IvfPqIndex::search
//     (crates/vector-index/src/ivf/mod.rs:277-284);
//   * KMeans::find_nearest_centroid (kmeans.rs:264-309): the one nearest
//     centroid of a vector, for every base vector while building the inverted
//     lists (mod.rs:119-125, 203-210) and in PQ training (pq.rs:190).
// Both are a flat kNN of the queries against the K centroids with the same
// pair arithmetic (the AVX-512 DistanceEngine), so they run on a vrs_knn
// handle created over the centroids: one batched search instead of a scalar
// loop per query. This file adds only the reference's result convention on
// top of that search:
//   * indices are widened to int64 (usize in the reference);
//   * the reference sorts by the reported value with a stable sort
//     (kmeans.rs:345-350), so exactly equal values keep index order. The kNN
//     engine orders by its ranking key, which for Minkowski, Mahalanobis and
//     Hellinger is the sum before the final root; two distinct sums can round
//     to the same root. For those metrics the search fetches a few extra
//     neighbours, re-orders runs of equal reported values by index and
//     truncates, widening the fetch when a run reaches its end;
//   * find_nearest_centroid's strict comparison (kmeans.rs:297-305) picks the
//     lowest index among equal best values, which is the first entry of that
//     order; with no centroids it returns index 0 and +inf (-inf for
//     similarities), the initial values of its loop (kmeans.rs:272-277).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "vrs_internal.cuh"

namespace {

// Queries per underlying search call: bounds the host staging of ids.
constexpr int64_t kProbeChunk = 1 << 16;
// Extra neighbours fetched for the metrics whose reported value is a root of
// the ranking key.
constexpr int kRootSlack = 8;
constexpr int kMaxFetch = 2048;  // the kNN engine's largest k'

bool rooted(int metric) {
  return metric == VRS_MINKOWSKI || metric == VRS_MAHALANOBIS || metric == VRS_HELLINGER;
}

int bad(const std::string& m) {
  vrs::set_error(VRS_ERR_INVALID_CONFIG, m);
  return VRS_ERR_INVALID_CONFIG;
}

// Top-p centroids of nb queries into score/idx (row stride p).
int probe_chunk(vrs_knn* h, int64_t K, int metric, const float* q, int64_t nb, int32_t p,
                float* score, int64_t* idx, std::vector<float>& dist, std::vector<uint32_t>& ids) {
  if (!rooted(metric)) {
    // The engine's order is already the reference's: search straight into the
    // caller's buffers, the u32 ids into the low half of out_idx, then widen
    // them in place from the last entry down (entry i's 8 bytes cover u32
    // slots 2i and 2i+1, both >= i, so both were read before i is written).
    uint32_t* ids32 = reinterpret_cast<uint32_t*>(idx);
    int32_t got = 0;
    int st = vrs_knn_search(h, q, nb, p, score, ids32, &got);
    if (st != VRS_OK) return st;
    if (got != p) return bad("ivf probe: search returned " + std::to_string(got) + " of " +
                             std::to_string(p) + " neighbours");
    // Byte copies: the buffer is read as u32 and written as i64 (no aliasing
    // of the two pointer types, and the compiler keeps each read before the
    // write that may cover it).
    char* raw = reinterpret_cast<char*>(idx);
    for (int64_t i = nb * (int64_t)p - 1; i >= 0; i--) {
      uint32_t v;
      memcpy(&v, raw + 4 * i, 4);
      const int64_t w = v;
      memcpy(raw + 8 * i, &w, 8);
    }
    return VRS_OK;
  }
  int32_t fetch = (int32_t)std::min<int64_t>({K, (int64_t)p + kRootSlack, kMaxFetch});
  for (;;) {
    dist.resize((size_t)nb * fetch);
    ids.resize((size_t)nb * fetch);
    int32_t got = 0;
    int st = vrs_knn_search(h, q, nb, fetch, dist.data(), ids.data(), &got);
    if (st != VRS_OK) return st;
    if (got != fetch) return bad("ivf probe: search returned " + std::to_string(got) + " of " +
                                 std::to_string(fetch) + " neighbours");
    // A run of equal reported values that reaches the last fetched entry may
    // continue past it: fetch more for the whole chunk (needs a run longer
    // than the slack at the probe boundary: duplicated centroids, or distinct
    // sums whose roots round equal).
    bool widen = false;
    if (fetch < K) {
      for (int64_t r = 0; r < nb && !widen; r++)
        widen = dist[r * fetch + fetch - 1] == dist[r * fetch + p - 1];
    }
    if (widen) {
      if (fetch >= kMaxFetch) return bad("ivf probe: a run of equal distances at the probe boundary "
                                         "is longer than the 2048 neighbours one search returns");
      fetch = (int32_t)std::min<int64_t>({K, (int64_t)fetch * 2, kMaxFetch});
      continue;
    }
    std::vector<int32_t> order(fetch);
    for (int64_t r = 0; r < nb; r++) {
      const float* dr = dist.data() + r * fetch;
      const uint32_t* ir = ids.data() + r * fetch;
      for (int j = 0; j < fetch; j++) order[j] = j;
      // Values are non-decreasing along the row (the root is monotone), so
      // ordering by (value, index) only reorders inside runs of equal values.
      std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
        return dr[a] < dr[b] || (dr[a] == dr[b] && ir[a] < ir[b]);
      });
      for (int j = 0; j < p; j++) {
        score[r * p + j] = dr[order[j]];
        idx[r * p + j] = ir[order[j]];
      }
    }
    return VRS_OK;
  }
}

}  // namespace

extern "C" int vrs_ivf_find_top_centroids(vrs_knn* centroids, const float* queries, int64_t nq,
                                          int32_t nprobe, float* out_score, int64_t* out_idx,
                                          int32_t* out_p) {
  if (!centroids || !out_p) return bad("vrs_ivf_find_top_centroids: null handle or out_p");
  *out_p = 0;
  if (nq < 0 || nprobe < 0) return bad("vrs_ivf_find_top_centroids: negative nq or nprobe");
  int64_t K = 0;
  int32_t d = 0, metric = 0;
  int st = vrs_knn_info(centroids, &K, &d, nullptr, nullptr, &metric);
  if (st != VRS_OK) return st;
  const int32_t p = (int32_t)std::min<int64_t>(nprobe, K);
  if (p == 0 || nq == 0) {
    *out_p = p;
    return VRS_OK;
  }
  if (p > kMaxFetch) return bad("vrs_ivf_find_top_centroids: nprobe' > 2048 is not supported");
  // The rooted metrics check the entry after the boundary for an equal root;
  // one search returns at most 2048, so P = 2048 < K leaves no room for it.
  if (rooted(metric) && p >= kMaxFetch && p < K)
    return bad("vrs_ivf_find_top_centroids: Minkowski, Mahalanobis and Hellinger support nprobe' <= 2047 "
               "when there are more centroids");
  if (!queries || !out_score || !out_idx) return bad("vrs_ivf_find_top_centroids: null buffer");
  std::vector<float> dist;
  std::vector<uint32_t> ids;
  for (int64_t q0 = 0; q0 < nq; q0 += kProbeChunk) {
    const int64_t nb = std::min(kProbeChunk, nq - q0);
    st = probe_chunk(centroids, K, metric, queries + q0 * d, nb, p, out_score + q0 * p,
                     out_idx + q0 * p, dist, ids);
    if (st != VRS_OK) return st;
  }
  *out_p = p;
  return VRS_OK;
}

extern "C" int vrs_ivf_assign(vrs_knn* centroids, const float* x, int64_t n, int64_t* out_idx,
                              float* out_score) {
  if (!centroids) return bad("vrs_ivf_assign: null handle");
  if (n < 0) return bad("vrs_ivf_assign: negative n");
  if (n == 0) return VRS_OK;
  if (!x || !out_idx) return bad("vrs_ivf_assign: null buffer");
  int64_t K = 0;
  int32_t d = 0, metric = 0;
  int st = vrs_knn_info(centroids, &K, &d, nullptr, nullptr, &metric);
  if (st != VRS_OK) return st;
  if (K == 0) {
    const float init = vrs_metric_higher_is_better(metric) == 1 ? -INFINITY : INFINITY;
    for (int64_t i = 0; i < n; i++) {
      out_idx[i] = 0;
      if (out_score) out_score[i] = init;
    }
    return VRS_OK;
  }
  std::vector<float> dist, score_tmp;
  std::vector<uint32_t> ids;
  if (!out_score) score_tmp.resize((size_t)std::min(kProbeChunk, n));
  for (int64_t q0 = 0; q0 < n; q0 += kProbeChunk) {
    const int64_t nb = std::min(kProbeChunk, n - q0);
    float* sc = out_score ? out_score + q0 : score_tmp.data();
    st = probe_chunk(centroids, K, metric, x + q0 * d, nb, 1, sc, out_idx + q0, dist, ids);
    if (st != VRS_OK) return st;
  }
  return VRS_OK;
}
