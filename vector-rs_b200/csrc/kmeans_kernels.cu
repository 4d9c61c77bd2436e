// kmeans_kernels.cu -- CUDA-core kernels of the Lloyd k-means path.
//   * kmeans_assign_exact: per point, the nearest centroid under the
//     reference's exact pair arithmetic (find_nearest,
//     crates/vector-cuda/src/kmeans.rs:361-407: strict comparison, lowest
//     index wins ties, argmax for dot/cosine);
//   * kmeans_accumulate: per-cluster sums as 64-bit fixed-point integers
//     (value * 2^s rounded), so the sum is exact, independent of the order
//     in which points arrive, and identical across GPUs after an integer
//     NCCL all-reduce; counts as 64-bit integers;
//   * kmeans_update: mean = (float)(sum / count) in f64, squared shift in f32
//     summed over dimensions in order (kmeans.rs:318-331); an empty cluster
//     keeps its centroid (reference kernel kernels/kmeans.cu:350-356);
//   * deterministic f64 reduction for the inertia; |x| maximum for the
//     fixed-point scale.
// Reference kernels replaced: kmeans_zero_accumulators,
// kmeans_assign_and_accumulate, kmeans_update_centroids
// (crates/vector-cuda/src/kernels/kmeans.cu:22-395).
#include <mutex>

#include "vrs_exact.cuh"
#include "vrs_internal.cuh"

namespace vrs {
namespace {

template <int METRIC>
__global__ void __launch_bounds__(128) kmeans_assign_exact_kernel(
    const float* __restrict__ x, int64_t n, int d, int dp, const float* __restrict__ cent,
    const float* __restrict__ cent_aux, const float* __restrict__ x_aux, int k,
    int32_t* __restrict__ assign, float* __restrict__ dist) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* v = x + i * dp;
  const float va = METRIC == vrs_exact::kCos ? x_aux[i] : 0.0f;
  const bool hib = vrs_exact::higher_is_better(METRIC);
  int best = 0;
  float best_key = hib ? -INFINITY : INFINITY;
  for (int c = 0; c < k; c++) {
    const float ca = METRIC == vrs_exact::kCos ? cent_aux[c] : 0.0f;
    float key = vrs_exact::rank_key(METRIC, v, cent + (int64_t)c * dp, d, va, ca);
    if (hib ? key > best_key : key < best_key) {
      best_key = key;
      best = c;
    }
  }
  assign[i] = best;
  dist[i] = vrs_exact::finish(METRIC, best_key);
}

__global__ void kmeans_accumulate_kernel(const float* __restrict__ x, int64_t n, int d, int dp,
                                         const int32_t* __restrict__ assign, int scale_exp,
                                         unsigned long long* __restrict__ sums,
                                         unsigned long long* __restrict__ counts) {
  // One warp per point: lanes stride over dimensions.
  int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (w >= n) return;
  int c = assign[w];
  const float* v = x + w * dp;
  unsigned long long* s = sums + (int64_t)c * dp;
  for (int j = lane; j < d; j += 32) {
    long long q = __double2ll_rn(ldexp((double)v[j], scale_exp));
    atomicAdd(&s[j], (unsigned long long)q);
  }
  if (lane == 0) atomicAdd(&counts[c], 1ull);
}

__global__ void kmeans_update_kernel(const unsigned long long* __restrict__ sums,
                                     const unsigned long long* __restrict__ counts, int k, int d,
                                     int dp, int scale_exp, float* __restrict__ cent,
                                     float* __restrict__ shift, float* __restrict__ max_shift) {
  int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= k) return;
  unsigned long long cnt = counts[c];
  if (cnt == 0) {
    shift[c] = 0.0f;
    return;
  }
  double inv_scale = ldexp(1.0, -scale_exp);
  float sh = 0.0f;
  for (int j = 0; j < d; j++) {
    double sum = (double)(long long)sums[(int64_t)c * dp + j] * inv_scale;
    float val = (float)(sum / (double)cnt);
    float old = cent[(int64_t)c * dp + j];
    float diff = __fsub_rn(val, old);
    sh = __fadd_rn(sh, __fmul_rn(diff, diff));
    cent[(int64_t)c * dp + j] = val;
  }
  shift[c] = sh;
  // Non-negative floats order like their bit patterns.
  atomicMax(reinterpret_cast<unsigned int*>(max_shift), __float_as_uint(sh));
}

// Warp per cluster: means in parallel, then the squared shift summed over
// dimensions in order (f32, separate multiply and add, kmeans.rs:318-331).
__global__ void kmeans_update_warp_kernel(const unsigned long long* __restrict__ sums,
                                          const unsigned long long* __restrict__ counts, int k, int d,
                                          int dp, int scale_exp, float* __restrict__ cent,
                                          float* __restrict__ shift, float* __restrict__ max_shift) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (c >= k) return;
  const unsigned long long cnt = counts[c];
  if (cnt == 0) {
    if (lane == 0) shift[c] = 0.0f;
    return;
  }
  const double inv_scale = ldexp(1.0, -scale_exp);
  float diff[8];
#pragma unroll
  for (int jj = 0; jj < 8; jj++) {
    const int j = jj * 32 + lane;
    diff[jj] = 0.0f;
    if (j < d) {
      const double sum = (double)(long long)sums[(int64_t)c * dp + j] * inv_scale;
      const float val = (float)(sum / (double)cnt);
      diff[jj] = __fsub_rn(val, cent[(int64_t)c * dp + j]);
      cent[(int64_t)c * dp + j] = val;
    }
  }
  float sh = 0.0f;
#pragma unroll
  for (int jj = 0; jj < 8; jj++) {
    if (jj * 32 >= d) break;
    for (int t = 0; t < 32; t++) {
      const float dj = __shfl_sync(0xffffffffu, diff[jj], t);
      if (jj * 32 + t < d) sh = __fadd_rn(sh, __fmul_rn(dj, dj));
    }
  }
  if (lane == 0) {
    shift[c] = sh;
    atomicMax(reinterpret_cast<unsigned int*>(max_shift), __float_as_uint(sh));
  }
}

__global__ void abs_max_kernel(const float* __restrict__ x, int64_t n, int d, int dp,
                               unsigned int* __restrict__ out) {
  float m = 0.0f;
  int64_t total = n * dp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int c = (int)(i % dp);
    if (c < d) m = fmaxf(m, fabsf(x[i]));
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// ---------------------------------------------- segmented centroid sums
// Points are bucketed by cluster (counting sort), then each chunk of at
// most kChunk points of one cluster is summed by one block in 64-bit fixed
// point and added to the cluster's sums with one integer atomic per
// dimension. Integer addition is associative, so the result does not
// depend on the order of points or blocks.
constexpr int kChunk = 256;

__global__ void km_count_kernel(const int32_t* __restrict__ assign, int64_t n, int* __restrict__ counts) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) atomicAdd(&counts[assign[i]], 1);
}

// Single block: exclusive scans of counts (point offsets) and of the chunk
// counts ceil(count / kChunk) (chunk offsets); zeroes the scatter cursors.
__global__ void km_scan_kernel(const int* __restrict__ counts, int k, int* __restrict__ off,
                               int* __restrict__ coff, int* __restrict__ cursor) {
  __shared__ int s_a[1024], s_b[1024];
  const int t = threadIdx.x;
  const int per = (k + 1023) / 1024;
  int a = 0, b = 0;
  for (int j = 0; j < per; j++) {
    int c = t * per + j;
    if (c < k) {
      a += counts[c];
      b += (counts[c] + kChunk - 1) / kChunk;
    }
  }
  s_a[t] = a;
  s_b[t] = b;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    int va = t >= o ? s_a[t - o] : 0, vb = t >= o ? s_b[t - o] : 0;
    __syncthreads();
    s_a[t] += va;
    s_b[t] += vb;
    __syncthreads();
  }
  int ra = s_a[t] - a, rb = s_b[t] - b;
  for (int j = 0; j < per; j++) {
    int c = t * per + j;
    if (c < k) {
      off[c] = ra;
      coff[c] = rb;
      cursor[c] = 0;
      ra += counts[c];
      rb += (counts[c] + kChunk - 1) / kChunk;
    }
  }
  if (t == 1023) {
    off[k] = s_a[t];
    coff[k] = s_b[t];
  }
}

// Block-local variants for k <= kSmemBins: a shared-memory histogram per
// block of kBinPts points, then one global atomic per non-empty bin (counts),
// or one range reservation per non-empty bin and local ranks (scatter).
constexpr int kSmemBins = 16384;
constexpr int kBinThreads = 256;
constexpr int kBinPer = 16;
constexpr int kBinPts = kBinThreads * kBinPer;

__global__ void __launch_bounds__(kBinThreads) km_count_smem_kernel(const int32_t* __restrict__ assign, int64_t n,
                                                                    int k, int* __restrict__ counts) {
  extern __shared__ int h[];
  for (int c = threadIdx.x; c < k; c += kBinThreads) h[c] = 0;
  __syncthreads();
  const int64_t b0 = (int64_t)blockIdx.x * kBinPts;
#pragma unroll
  for (int u = 0; u < kBinPer; u++) {
    const int64_t i = b0 + u * kBinThreads + threadIdx.x;
    if (i < n) atomicAdd(&h[assign[i]], 1);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < k; c += kBinThreads)
    if (h[c]) atomicAdd(&counts[c], h[c]);
}

__global__ void __launch_bounds__(kBinThreads) km_scatter_smem_kernel(const int32_t* __restrict__ assign, int64_t n,
                                                                      int k, const int* __restrict__ off,
                                                                      int* __restrict__ cursor,
                                                                      int32_t* __restrict__ perm) {
  extern __shared__ int h[];
  for (int c = threadIdx.x; c < k; c += kBinThreads) h[c] = 0;
  __syncthreads();
  const int64_t b0 = (int64_t)blockIdx.x * kBinPts;
  int cl[kBinPer], lr[kBinPer];
#pragma unroll
  for (int u = 0; u < kBinPer; u++) {
    const int64_t i = b0 + u * kBinThreads + threadIdx.x;
    cl[u] = i < n ? assign[i] : -1;
    lr[u] = cl[u] >= 0 ? atomicAdd(&h[cl[u]], 1) : 0;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < k; c += kBinThreads) {
    const int cnt = h[c];
    h[c] = cnt ? off[c] + atomicAdd(&cursor[c], cnt) : 0;
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kBinPer; u++)
    if (cl[u] >= 0) perm[h[cl[u]] + lr[u]] = (int32_t)(b0 + u * kBinThreads + threadIdx.x);
}

__global__ void km_scatter_kernel(const int32_t* __restrict__ assign, int64_t n, const int* __restrict__ off,
                                  int* __restrict__ cursor, int32_t* __restrict__ perm) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) {
    const int c = assign[i];
    perm[off[c] + atomicAdd(&cursor[c], 1)] = (int32_t)i;
  }
}

// One block (4 warps) per chunk; lane l of a warp owns dimensions l + 32 j.
template <int NJ>
__global__ void __launch_bounds__(128) km_chunk_sum_kernel(
    const float* __restrict__ x, int d, int dp, int k, const int* __restrict__ off,
    const int* __restrict__ coff, const int32_t* __restrict__ perm, int scale_exp,
    unsigned long long* __restrict__ sums) {
  __shared__ long long s_part[4][NJ * 32];
  const int b = blockIdx.x;
  if (b >= coff[k]) return;
  int lo = 0, hi = k;  // cluster c with coff[c] <= b < coff[c+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (coff[mid] <= b) lo = mid; else hi = mid;
  }
  const int c = lo;
  const int p0 = off[c] + (b - coff[c]) * kChunk;
  const int p1 = min(off[c + 1], p0 + kChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long acc[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++) acc[j] = 0;
  // v * 2^s is exact in f32 (|v| 2^s < 2^61; a product that underflows is
  // below 1/2 and rounds to 0 either way), so f32 -> s64 rounding gives the
  // same integer as the f64 path at a fraction of the cost.
  const float scalef = ldexpf(1.0f, scale_exp);
  // Four points per warp step (indices, then all their rows, in flight
  // together): the rows are scattered, so memory-level parallelism is what
  // sets the rate.
  constexpr int U = 4;
  for (int p = p0 + warp * U; p < p1; p += 4 * U) {
    int64_t row[U];
#pragma unroll
    for (int u = 0; u < U; u++) row[u] = p + u < p1 ? (int64_t)perm[p + u] : -1;
    float val[U][NJ];
#pragma unroll
    for (int u = 0; u < U; u++)
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const int e = lane + 32 * j;
        val[u][j] = (row[u] >= 0 && e < d) ? x[row[u] * dp + e] : 0.0f;
      }
#pragma unroll
    for (int u = 0; u < U; u++)
#pragma unroll
      for (int j = 0; j < NJ; j++) acc[j] += __float2ll_rn(val[u][j] * scalef);
  }
#pragma unroll
  for (int j = 0; j < NJ; j++) s_part[warp][lane + 32 * j] = acc[j];
  __syncthreads();
  for (int e = threadIdx.x; e < d; e += 128) {
    const long long t = s_part[0][e] + s_part[1][e] + s_part[2][e] + s_part[3][e];
    if (t) atomicAdd(&sums[(int64_t)c * dp + e], (unsigned long long)t);
  }
}

__global__ void km_counts_u64_kernel(const int* __restrict__ counts, int k, unsigned long long* __restrict__ out) {
  int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < k) out[c] = (unsigned long long)counts[c];
}

constexpr int kSumBlocks = 512;
constexpr int kSumThreads = 256;

// Deterministic f64 sum: fixed partition of indices over a fixed grid, fixed
// in-block tree, then one block sums the partials in a fixed tree.
__global__ void sum_f64_stage1(const float* __restrict__ v, int64_t n, double* __restrict__ part) {
  __shared__ double s[kSumThreads];
  double acc = 0.0;
  for (int64_t i = blockIdx.x * (int64_t)kSumThreads + threadIdx.x; i < n;
       i += (int64_t)kSumBlocks * kSumThreads)
    acc = __dadd_rn(acc, (double)v[i]);
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kSumThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) s[threadIdx.x] = __dadd_rn(s[threadIdx.x], s[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = s[0];
}

__global__ void sum_f64_stage2(double* __restrict__ part, double* __restrict__ out) {
  __shared__ double s[kSumBlocks];
  for (int i = threadIdx.x; i < kSumBlocks; i += blockDim.x) s[i] = part[i];
  __syncthreads();
  for (int w = kSumBlocks / 2; w > 0; w >>= 1) {
    for (int i = threadIdx.x; i < w; i += blockDim.x) s[i] = __dadd_rn(s[i], s[i + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = s[0];
}

template <int M>
struct AssignL {
  static int run(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
                 const float* x_aux, int k, int32_t* assign, float* dist, cudaStream_t s) {
    kmeans_assign_exact_kernel<M><<<(unsigned)((n + 127) / 128), 128, 0, s>>>(
        x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist);
    VRS_CUDA(cudaGetLastError());
    count_launch();
    return VRS_OK;
  }
};

}  // namespace

int launch_kmeans_assign_exact(const float* x, int64_t n, int d, int dp, const float* cent,
                               const float* cent_aux, const float* x_aux, int k, int metric,
                               int32_t* assign, float* dist, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  switch (metric) {
    case 0: return AssignL<0>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 1: return AssignL<1>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 2: return AssignL<2>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 3: return AssignL<3>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 4: return AssignL<4>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 5: return AssignL<5>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 6: return AssignL<6>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 7: return AssignL<7>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 8: return AssignL<8>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
    case 9: return AssignL<9>::run(x, n, d, dp, cent, cent_aux, x_aux, k, assign, dist, s);
  }
  set_error(VRS_ERR_INVALID_CONFIG, "unknown metric");
  return VRS_ERR_INVALID_CONFIG;
}

int launch_kmeans_accumulate(const float* x, int64_t n, int d, int dp, const int32_t* assign, int k,
                             int scale_exp, unsigned long long* sums, unsigned long long* counts,
                             cudaStream_t s) {
  (void)k;
  if (n == 0) return VRS_OK;
  int64_t threads = n * 32;
  kmeans_accumulate_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
      x, n, d, dp, assign, scale_exp, sums, counts);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

int launch_kmeans_segsum(const float* x, int64_t n, int d, int dp, const int32_t* assign, int k,
                         int scale_exp, unsigned long long* sums, unsigned long long* counts, int* ws,
                         cudaStream_t s) {
  if (n == 0) return VRS_OK;
  if (d > 256) return launch_kmeans_accumulate(x, n, d, dp, assign, k, scale_exp, sums, counts, s);
  int* cnt = ws;                // [k]
  int* off = cnt + k;           // [k+1]
  int* coff = off + k + 1;      // [k+1]
  int* cursor = coff + k + 1;   // [k]
  int32_t* perm = cursor + k;   // [n]
  VRS_CUDA(cudaMemsetAsync(cnt, 0, (size_t)k * sizeof(int), s));
  const unsigned nb = (unsigned)((n + 255) / 256);
  const bool smem_bins = k <= kSmemBins;
  if (smem_bins) {
    static std::once_flag once[64];
    int dev = 0;
    VRS_CUDA(cudaGetDevice(&dev));
    auto set = [] {
      cudaFuncSetAttribute(km_count_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBins * 4);
      cudaFuncSetAttribute(km_scatter_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBins * 4);
    };
    if (dev < 64)
      std::call_once(once[dev], set);
    else
      set();
  }
  const unsigned nbb = (unsigned)((n + kBinPts - 1) / kBinPts);
  const size_t hsm = (size_t)k * sizeof(int);
  if (smem_bins)
    km_count_smem_kernel<<<nbb, kBinThreads, hsm, s>>>(assign, n, k, cnt);
  else
    km_count_kernel<<<nb, 256, 0, s>>>(assign, n, cnt);
  km_scan_kernel<<<1, 1024, 0, s>>>(cnt, k, off, coff, cursor);
  if (smem_bins)
    km_scatter_smem_kernel<<<nbb, kBinThreads, hsm, s>>>(assign, n, k, off, cursor, perm);
  else
    km_scatter_kernel<<<nb, 256, 0, s>>>(assign, n, off, cursor, perm);
  const unsigned nchunks = (unsigned)((n + kChunk - 1) / kChunk + k);
  if (d <= 128)
    km_chunk_sum_kernel<4><<<nchunks, 128, 0, s>>>(x, d, dp, k, off, coff, perm, scale_exp, sums);
  else
    km_chunk_sum_kernel<8><<<nchunks, 128, 0, s>>>(x, d, dp, k, off, coff, perm, scale_exp, sums);
  km_counts_u64_kernel<<<(k + 255) / 256, 256, 0, s>>>(cnt, k, counts);
  VRS_CUDA(cudaGetLastError());
  count_launch(5);
  return VRS_OK;
}

size_t kmeans_segsum_ws_bytes(int64_t n, int k) { return ((size_t)4 * k + 2 + (size_t)n) * sizeof(int); }

int launch_kmeans_update(const unsigned long long* sums, const unsigned long long* counts, int k,
                         int d, int dp, int scale_exp, float* cent, float* shift, float* max_shift,
                         cudaStream_t s) {
  VRS_CUDA(cudaMemsetAsync(max_shift, 0, sizeof(float), s));
  if (d <= 256)
    kmeans_update_warp_kernel<<<(unsigned)(((int64_t)k * 32 + 127) / 128), 128, 0, s>>>(
        sums, counts, k, d, dp, scale_exp, cent, shift, max_shift);
  else
    kmeans_update_kernel<<<(k + 127) / 128, 128, 0, s>>>(sums, counts, k, d, dp, scale_exp, cent,
                                                         shift, max_shift);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

int launch_abs_max(const float* x, int64_t n, int d, int dp, float* out, cudaStream_t s) {
  VRS_CUDA(cudaMemsetAsync(out, 0, sizeof(float), s));
  if (n == 0) return VRS_OK;
  abs_max_kernel<<<148 * 8, 256, 0, s>>>(x, n, d, dp, reinterpret_cast<unsigned int*>(out));
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

// out must have room for kSumBlocks + 1 doubles; the sum lands in out[kSumBlocks].
int launch_sum_f64(const float* v, int64_t n, double* out, cudaStream_t s) {
  sum_f64_stage1<<<kSumBlocks, kSumThreads, 0, s>>>(v, n, out);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  sum_f64_stage2<<<1, 256, 0, s>>>(out, out + kSumBlocks);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

}  // namespace vrs
