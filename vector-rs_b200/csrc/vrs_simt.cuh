// vrs_simt.cuh -- host-side interface of the CUDA-core scan (knn_simt.cu)
// for Manhattan, Chebyshev and Hellinger.
#pragma once
#include "vrs_internal.cuh"

namespace vrs {
namespace simt {

constexpr int kSimtMaxDp = 128;  // padded dimension held in shared memory

struct SimtPlan {
  int qtiles;       // CTAs along the queries (128 each)
  int nseg;         // base segments (one candidate list per segment and query)
  int64_t seg_len;  // rows per segment, a multiple of the 128-row tile
};

bool simt_supported(int metric, int dp);
// Bound slack of the scan's scores against the reference-order scores:
// rows with scan score <= tau * rho keep every exact top-k row.
float simt_rho(int metric, int d);
SimtPlan simt_plan(int64_t n, int nq, int num_sms);
// Scans rows base[i * stride] (i < n): appends (score, i) with score <=
// init_bound[q] to the lists, or, with tmin != null, writes each 128-row
// tile's minimum per query to tmin[q * tmin_stride + tile].
int simt_scan(const float* base, int64_t n, int64_t stride, int dp, const float* q, int nq, int metric,
              const SimtPlan& p, Cand* cand, int* cnt, int* overflow, int cap, const float* init_bound, float* tmin,
              int64_t tmin_stride, cudaStream_t s);
// init_bound[q] = (k-th smallest of tmin[q][0..ntile)) * rho, rounded up
// (+inf when ntile < k).
int simt_tau(const float* tmin, int ntile, int nq, int k, float rho, float* init_bound, cudaStream_t s);
int64_t simt_tile_rows();
// Pivot set of a search with k neighbours: every *stride-th row of a shard
// of n rows (`parts` shards share the base); returns its row count.
int64_t simt_pivot_rows(int64_t n, int k, int parts, int64_t* stride);

}  // namespace simt
}  // namespace vrs
