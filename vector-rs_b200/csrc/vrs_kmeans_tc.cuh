// vrs_kmeans_tc.cuh -- host-side interface of the tensor-core k-means
// assignment (kmeans_tc.cu).
#pragma once
#include "vrs_internal.cuh"

namespace vrs {
namespace kmtc {

// Per (point, column half) result of the tensor-core pass: approximate best
// score and centroid, number of kept candidates (at most 8, the best within
// the margin), and the smallest score that did not fit (+inf if none).
struct Res {
  float best;
  uint32_t bi;
  int cnt;
  float lost;
};

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
           const unsigned int* cmax, int metric, float op_scale, Res* res, Cand* cands, int* err, int num_sms,
           const float* init_bound, cudaStream_t s);
// Exact assignment from the candidates (flags: 2 n + 2 ints of scratch).
// Points whose candidates may be incomplete are assigned by a full exact
// scan, one CTA per point; points with several candidates within their
// bound by exact scoring of those; a point with a single candidate within
// its bound takes it and gets no exact distance here (fill_dist).
int finalize(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
             const float* x_aux, int k, const float* xq, const unsigned int* cmax, int metric, const Res* res,
             const Cand* cands, const int* force_full, int32_t* assign_out, float* dist, int* flags, int num_sms,
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
