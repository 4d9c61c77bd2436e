// vrs_internal.cuh -- shared device helpers and host-side error plumbing for
// libvrs (not part of the public ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/vrs.h"

namespace vrs {

// ---------------------------------------------------------------- errors
void set_error(int status, const std::string& msg);
int cuda_status(cudaError_t e);  // maps a CUDA error to a vrs status

#define VRS_CUDA(call)                                                            \
  do {                                                                            \
    cudaError_t _e = (call);                                                      \
    if (_e != cudaSuccess) {                                                      \
      ::vrs::set_error(::vrs::cuda_status(_e), std::string(#call) + ": " +        \
                                                   cudaGetErrorString(_e));       \
      return ::vrs::cuda_status(_e);                                              \
    }                                                                             \
  } while (0)

#define VRS_TRY(expr)          \
  do {                         \
    int _s = (expr);           \
    if (_s != VRS_OK) return _s; \
  } while (0)

// ---------------------------------------------------------- profiling
// Optional CUDA-event timing of named launches (profile.cu).
struct ProfToken {
  bool active = false;
  const char* name = nullptr;
  int device = 0;
  cudaEvent_t start = nullptr, stop = nullptr;
};
ProfToken prof_begin(const char* name, cudaStream_t s);
void prof_end(ProfToken& t, cudaStream_t s);
// Counts kernel launches issued by this library (read as profile name "*").
void count_launch(int n = 1);
// Adds n to the count of a named event (read back as the "launches" of
// vrs_profile_read(name); total_ms stays 0); only while every stage is timed.
void prof_count(const char* name, int64_t n);

// ------------------------------------------------------- candidate lists
// One candidate of a per-(segment, query) list: heap score (smaller is
// better; similarities are negated) and the row index inside the shard.
struct Cand {
  float hs;
  uint32_t id;
};

// Merge-pair id that marks "rows of this shard at or beyond this score may
// be missing" (ids are below 2^32 - 2; 0xffffffff is padding). A query whose
// merged top-k' holds one is searched again exactly.
constexpr uint32_t kSentinelId = 0xfffffffeu;

// Monotone map float -> uint32 (total order of non-NaN floats).
__host__ __device__ __forceinline__ uint32_t ord_key(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ __forceinline__ float ord_inv(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// How a scan's scores relate to the exact (reference-order) scores.
enum ScanKind : int {
  kExactScores = 0,  // scan scores are the exact heap scores
  kRelMargin = 1,    // non-negative sums: exact <= approx * rho and vice versa
  kAbsMargin = 2,    // |approx - exact| <= margin[q] / 2 per query
};

// Acceptance bound from the running k-th best approximate score tau: every
// row that could still belong to the exact top-k has approx <= bound.
__device__ __forceinline__ float accept_bound(int kind, float tau, float rho, float absm) {
  if (kind == kRelMargin) return __fmul_ru(tau, rho);
  if (kind == kAbsMargin) return __fadd_ru(tau, absm);
  return tau;
}

struct KnnScanArgs {
  const float* base;     // [n][dp] row-major (Hellinger: per-element roots)
  const float* base_aux; // per-row aux (cosine: norm^2 in the cosine order)
  int64_t n;             // rows in this shard
  int d, dp;
  const float* q;        // [nq][dp] (Hellinger: roots)
  const float* q_aux;    // per-query aux
  const int* q_index;    // optional map slot -> query row (fallback re-runs)
  int nq;
  int k;
  int64_t seg_len;
  int nseg;
  Cand* cand;            // [nseg][nq][cap]
  int* cnt;              // [nseg][nq]
  int* overflow;         // [nq]
  int cap;
  int metric;
  int kind;
  float rho;
  const float* absm;     // [nq] (kAbsMargin)
};

struct KnnSelectArgs {
  const float* base;     // exact re-rank operands (as in KnnScanArgs)
  const float* base_aux;
  int d, dp;
  const float* q;
  const float* q_aux;
  const int* q_index;
  int nq;
  int k;                 // k' (results per query)
  int nseg;
  const Cand* cand;
  const int* cnt;
  int* overflow;
  int cap;
  int metric;
  int kind;
  float rho;
  const float* absm;
  uint32_t id_offset;    // global id of shard row 0
  // outputs: either final (dist, id) or merge pairs (hs, global id)
  float* out_dist;       // [nq][k] or null
  uint32_t* out_id;      // [nq][k] or null
  Cand* out_pairs;       // [nq][k] or null
  int max_sort;          // shared-memory sort capacity (power of two)
  const uint32_t* tiny;  // rows always re-ranked exactly (cosine near-zero rows)
  int n_tiny;
  int retry;             // block select: only the slots the warp select flagged (2)
  // Starting acceptance bound of the scan per slot when it was not proven to
  // cover k rows (null otherwise). The select then checks that the scan kept
  // at least k rows and that the k-th best kept score plus the margin stays
  // within it; a slot that fails goes to the exact fallback (overflow 1).
  const float* init_bound;
  // With init_bound and merge pairs: a slot whose bound fails the check is
  // not flagged; its pairs keep the rows scored below init_bound - absm / 2
  // (no unkept row of this shard can score below that) followed by a
  // kSentinelId pair at that score, and the merge decides.
  int certify;
  // Squared L2 / Mahalanobis: per query row a lower bound of |q|^2. The
  // scan's scores (|x|^2 - 2 q.x) leave it out and the exact heap scores
  // include it, so the certified limit above is moved by it before it is
  // compared with exact scores (null: no offset).
  const float* q_sq;
};

// Launchers (knn_kernels.cu).
int launch_knn_scan_exact(const KnnScanArgs& a, cudaStream_t s);
int launch_knn_select(const KnnSelectArgs& a, cudaStream_t s);
// Warp-per-query select with half-warp exact re-rank (approximate scans of
// L2 / Mahalanobis / dot / cosine; nseg <= 32, k <= 512).
int launch_knn_select_warp(const KnnSelectArgs& a, cudaStream_t s);
// flags (nullable, [nq]) is set to 1 for queries whose merged top-k' holds
// a kSentinelId pair.
int launch_merge_pairs(const Cand* gathered, int nlists, int nq, int k, int metric,
                       float* out_dist, uint32_t* out_id, int* flags, cudaStream_t s);
// Slots with overflow != 0 get pairs (-inf, kSentinelId), then padding, so
// that the merge flags them.
int launch_flag_pairs(const int* overflow, int nq, int k, Cand* pairs, cudaStream_t s);
// dst[idx[i]] = src[i] for i < n.
int launch_scatter_flags(const int* src, const int* idx, int n, int* dst, cudaStream_t s);
int launch_pad_rows(const float* src, int64_t rows, int d, int dp, float* dst, int transform,
                    cudaStream_t s);
int launch_cos_norms(const float* x, int64_t rows, int d, int dp, float* out, cudaStream_t s);
int launch_finish_pairs(const Cand* pairs, int64_t count, int metric, float* out_dist,
                        uint32_t* out_id, cudaStream_t s);

// k-means launchers (kmeans_kernels.cu).
int launch_kmeans_assign_exact(const float* x, int64_t n, int d, int dp, const float* cent,
                               const float* cent_aux, const float* x_aux, int k, int metric,
                               int32_t* assign, float* dist, cudaStream_t s);
int launch_kmeans_accumulate(const float* x, int64_t n, int d, int dp, const int32_t* assign,
                             int k, int scale_exp, unsigned long long* sums,
                             unsigned long long* counts, cudaStream_t s);
// Deterministic per-cluster fixed-point sums through a counting sort (d <= 256;
// larger d falls back to per-element integer atomics). ws: kmeans_segsum_ws_bytes.
int launch_kmeans_segsum(const float* x, int64_t n, int d, int dp, const int32_t* assign, int k,
                         int scale_exp, unsigned long long* sums, unsigned long long* counts, int* ws,
                         cudaStream_t s);
size_t kmeans_segsum_ws_bytes(int64_t n, int k);
int launch_kmeans_update(const unsigned long long* sums, const unsigned long long* counts,
                         int k, int d, int dp, int scale_exp, float* cent, float* shift,
                         float* max_shift, cudaStream_t s);
int launch_abs_max(const float* x, int64_t n, int d, int dp, float* out, cudaStream_t s);
int launch_sum_f64(const float* v, int64_t n, double* out, cudaStream_t s);

// Generator launcher (gen_kernels.cu).
int launch_gen_rows(int kind, uint64_t seed, uint32_t stream, int64_t row0, int64_t rows, int d,
                    int ld, float* out, const float* centres, uint32_t K, double sigma,
                    cudaStream_t s);

}  // namespace vrs
