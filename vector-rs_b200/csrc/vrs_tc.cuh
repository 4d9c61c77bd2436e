// vrs_tc.cuh -- host-side interface of the tensor-core scan (knn_tc.cu).
#pragma once
#include <cmath>

#include "vrs_internal.cuh"

namespace vrs {
namespace tc {

// Cosine rows or queries whose norm is below this go through the exact
// path: for every other pair sqrt(|q|^2) * sqrt(|x|^2) >= 1e-8 > 1e-9, so
// the reference's zero guard (crates/vector-simd/src/avx512.rs:218-221)
// never fires on the tensor-core path.
constexpr float kTinyNorm = 1e-4f;
constexpr int kTinyCap = 2048;

// Each segment keeps two candidate lists per query (one per column half of
// every tile), so a plan with nseg segments has 2 * nseg lists per query.
struct TcPlan {
  int qtiles;
  int nseg;
  int64_t seg_len;
  int cap;
};

bool tc_supported(int metric, int d);
// Squared L2 / Mahalanobis with d <= 126 fold -|x|^2 / 2 into the GEMM as two
// extra K columns (hi + lo fp16 of -xscale |x|^2 / 2^(m+1); the query side
// holds qscale * 2^m in both).
__host__ __device__ inline bool tc_fold(int metric, int d) {
  return (metric == 0 || metric == 7) && d + 2 <= 128;  // kL2, kMaha
}
// Operands go to the tensor cores as fp16 (11 significant bits; bf16's 8
// would make the error margin 8x wider): cosine rows unit-normalised, the
// other metrics scaled by powers of two (base: largest element in [2^7, 2^8);
// each query likewise), undone exactly in the epilogue.
__host__ __device__ inline bool tc_fp16(int) { return true; }
// Operand row length (multiple of 16): d, plus the folded columns.
int tc_d16(int metric, int d);
// xscale: the base's operand scale; fold_m: exponent of the folded -|x|^2
// column (tc_fold_exponent).
int tc_base_prep(const float* x, int64_t n, int d, int dp, int metric, float xscale, int fold_m, void* xb,
                 float* xn, unsigned int* xmax_bits, uint32_t* tiny, int* n_tiny, int tiny_cap, cudaStream_t s);
// From the unpadded queries q_in ([nq][d]): the padded f32 rows qpad
// ([nq][dp], for the exact re-rank), cosine norms in the reference's order
// (qaux, cosine only), fp16 operand rows, each query's operand scale
// (qscale) and margin (absm), and (qsq, nullable) a lower bound of |q|^2 in
// f32. Near-zero cosine queries and queries whose scale cannot fit the
// folded column are flagged for the exact scan.
int tc_query_prep(const float* q_in, int nq, int d, int dp, int metric, const unsigned int* xmax_bits,
                  float xscale, int fold_m, float* qpad, float* qaux, void* qb, float* qscale, float* absm,
                  int* overflow, float* qsq, cudaStream_t s);
// Base operand scale for a base whose largest |element| is maxabs, and the
// folded column's exponent (|F| = xscale |x|^2 / 2^(m+1) <= 2^14 with
// |x|^2 <= d maxabs^2).
inline float tc_base_scale(int metric, float maxabs) {
  if (metric == 2 || !(maxabs > 0.0f) || !std::isfinite(maxabs)) return 1.0f;  // kCos: unit rows
  int ex = 7 - std::ilogb(maxabs);
  ex = ex < -60 ? -60 : (ex > 60 ? 60 : ex);
  return std::ldexp(1.0f, ex);
}
inline int tc_fold_exponent(int d, float xscale, float maxabs) {
  if (!(maxabs > 0.0f)) return 0;
  const double top = (double)xscale * d * (double)maxabs * (double)maxabs;
  return (int)std::ceil(std::log2(top)) - 15;
}
// align_tiles: segments hold a multiple of this many 128-row tiles (the
// pivot pass passes kPivotGroup).
TcPlan tc_plan(int64_t n, int nq, int kk, int num_sms, int align_tiles = 1);
// The scan on CTA pairs (cta_group::2, M = N = 256): its plan and launch;
// its lists are [4 * nseg][nq][cap] (one per 64-column quarter). With tmin
// != null it is the pivot pass (plan aligned to kPivotGroup tiles), writing
// tc_pivot_values2(n) minima per query.
TcPlan tc_plan2(int64_t n, int nq, int kk, int num_sms, int align_tiles = 1);
int tc_scan2(const void* qb, int nq_rows_alloc, const void* xb, int64_t n, int d, const float* xn, int metric,
             int nq, int kk, const TcPlan& p, Cand* cand, int* cnt, int* overflow, const float* absm, int* err,
             float* tmin, const float* init_bound, const float* qscale, float xscale, cudaStream_t s);
// The pivot pass reports one minimum per column half of every group of
// kPivotGroup 128-row tiles (256 pivot rows per value): fewer values to
// store and to select from, each still the score of a distinct row.
constexpr int kPivotGroup = 4;
inline int64_t tc_pivot_groups(int64_t m) { return ((m + 127) / 128 + kPivotGroup - 1) / kPivotGroup; }
// Minima per query of the pair kernel's pivot pass: four 64-column quarters
// of every group of kPivotGroup 256-row tiles (256 rows per value).
inline int64_t tc_pivot_values2(int64_t m) { return 4 * (((m + 255) / 256 + kPivotGroup - 1) / kPivotGroup); }
// With tmin != null this is the pivot pass (per-tile minima, no appends);
// init_bound (nullable) seeds each query's acceptance bound.
int tc_scan(const void* qb, int nq_rows_alloc, const void* xb, int64_t n, int d, const float* xn,
            int metric, int nq, int kk, const TcPlan& p, Cand* cand, int* cnt, int* overflow,
            const float* absm, int* err, float* tmin, const float* init_bound, const float* qscale, float xscale,
            cudaStream_t s);
int tc_pivot_gather(const void* xb, const float* xn, int64_t m, int64_t stride, int d16, void* pb,
                    float* pn, cudaStream_t s);
// Starting bound per query from pivot minima: query q's values are
// vals[p * part_stride + q * len + j] for p < nparts, j < len (one part per
// shard after an all-gather, or nparts = 1 for a single shard's minima); the
// bound is the k-th smallest of them plus absm[q].
int tc_tau(const float* vals, int nparts, int64_t part_stride, int len, int nq, int k, const float* absm,
           float* init_bound, cudaStream_t s);
// The k smallest of each query's ntile pivot minima (query-major rows) into
// out[q * k + j], padded with +inf when there are fewer than k.
int tc_pivot_topk(const float* tmin, int ntile, int nq, int k, float* out, cudaStream_t s);
// Rank of the pivot minimum that seeds an unproven starting bound (one
// shard, pivot set = every stride-th row, so a row is a pivot row with
// probability p = 1/stride). Below the j-th pivot minimum lie about j/p base
// rows, with standard deviation sqrt(j (1 - p))/p; j is the smallest rank
// whose count stays at k or more 4.5 standard deviations below the mean. The
// select verifies the bound per query (k rows kept, k-th kept score plus
// margin within it) and sends a query that fails to the exact fallback. Never
// above k, where the bound is proven.
inline int tc_optimistic_rank(int k, int64_t stride) {
  if (stride <= 1) return k;
  const double p = 1.0 / (double)stride, z = 4.5;
  for (int j = 1; j < k; j++)
    if (j - z * std::sqrt(j * (1.0 - p)) >= k * p) return j;
  return k;
}

// Rows in the pivot set (every stride-th row) of a shard of n rows when
// `parts` shards share one base and pool their pivot minima: the pooled
// pivot set is about 1/6 of the base and at least 65,536 rows; beyond
// 1.6M pivot rows, 1/16 of the shard (the pivot pass's epilogue is cheap, and
// a denser pivot keeps the candidate band of huge bases small).
inline int64_t tc_pivot_rows(int64_t n, int parts, int64_t* stride) {
  int64_t m = n / 6;
  const int64_t lo = (65536 + parts - 1) / parts;
  if (m < lo) m = lo;
  const int64_t hi = n / 16 > 1600000 ? n / 16 : 1600000;
  if (m > hi) m = hi;
  if (m >= n) {
    *stride = 1;
    return n;
  }
  *stride = n / m;
  return n / *stride;
}

}  // namespace tc
}  // namespace vrs
