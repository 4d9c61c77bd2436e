// vrs_kmeans_tc.cuh -- host-side interface of the tensor-core k-means
// assignment (kmeans_tc.cu).
#pragma once
#include "vrs_internal.cuh"

namespace vrs {
namespace kmtc {

// Per (point, column half) result of the tensor-core pass: approximate best
// score, number of kept candidate groups (at most kGroupSlots), and the
// smallest group minimum that did not fit (+inf if none).
struct Res {
  float best;
  uint32_t bi;  // unused
  int cnt;
  float lost;
};

// Candidate groups: the pass keeps, per (point, column half), up to
// kGroupSlots groups of four consecutive centroids whose smallest
// approximate score was within the point's bound when seen: their four
// scores (sc) and first centroid index (col). Record r = 2 * point + half
// owns slots [r * kGroupSlots, (r + 1) * kGroupSlots). One allocation of
// group_bytes(n) holds both arrays.
constexpr int kGroupSlots = 8;
struct Groups {
  float4* sc;
  uint32_t* col;
};
inline size_t group_bytes(int64_t n) {
  return (size_t)n * 2 * kGroupSlots * (sizeof(float4) + sizeof(uint32_t));
}
inline Groups groups_at(void* base, int64_t n) {
  Groups g;
  g.sc = static_cast<float4*>(base);
  g.col = reinterpret_cast<uint32_t*>(static_cast<char*>(base) + (size_t)n * 2 * kGroupSlots * sizeof(float4));
  return g;
}

bool supported(int metric, int d);
// fp16 operand rows, |row|^2 (sq, nullable), |row| (nrm, nullable), max |row|
// (maxn, nullable), near-zero cosine flags (nullable).
// Operands are fp16 of value * op_scale (a power of two putting the largest
// element of points and centroids in [2^13, 2^14); 1 for cosine, whose rows
// are normalised). sq / nrm / maxn are unscaled.
int prep_rows(const float* x, int64_t n, int d, int dp, int metric, float op_scale, void* xb, float* sq,
              float* nrm, unsigned int* maxn, int* tiny_flag, int* any_tiny, cudaStream_t s);
// init_bound (nullable; squared L2 / Mahalanobis only): per point an upper
// bound on some centroid's score |c|^2 - 2 x.c (start_bound).
int assign(const void* xb, int64_t n, const void* cb, int k, int d, const float* cn, const float* xq,
           const unsigned int* cmax, int metric, float op_scale, Res* res, void* groups, int* err, int num_sms,
           const float* init_bound, cudaStream_t s);
// Exact assignment from the candidate groups (groups: as written by assign
// for the same n; flags: 2 n + 2 ints of scratch).
// Points whose candidates may be incomplete are assigned by a full exact
// scan, one CTA per point; points with several candidates within their
// bound by exact scoring of those; a point with a single candidate within
// its bound takes it and gets no exact distance here (fill_dist).
int finalize(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
             const float* x_aux, int k, const float* xq, const unsigned int* cmax, int metric, const Res* res,
             void* groups, const int* force_full, int32_t* assign_out, float* dist, int* flags, int num_sms,
             float op_scale, float* pscore, cudaStream_t s);
// pscore (written by finalize, squared L2 / Mahalanobis; +inf for points
// scanned exactly): an upper bound on each point's score to the centroid it
// was assigned. start_bound turns it into the next step's init_bound with the
// update's per-centroid squared shifts.
int start_bound(int64_t n, const int32_t* assign, const float* pscore, const float* xq, const float* shift,
                float* out, cudaStream_t s);
// dist[i] = exact distance of point i to centroid assign[i] (the centroids
// the assignment was made against), in the reference's arithmetic.
int fill_dist(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
              const float* x_aux, int metric, const int32_t* assign, float* dist, cudaStream_t s);

}  // namespace kmtc
}  // namespace vrs
