// knn_simt.cu -- CUDA-core scan for the non-GEMM metrics of the flat kNN
// path: Manhattan (L1), Chebyshev (L-inf) and Hellinger (squared L2 of
// per-element square roots, stored by the row layout kernels).
//
// A CTA scores 128 queries against 128-row tiles of one base segment. Each
// of its 256 threads accumulates an 8 x 8 (query, row) block in registers:
// per dimension a subtraction and an |.|-add (L1), a |.|-max (L-inf) or an
// FMA of the square (Hellinger). Queries stay in shared memory for the whole
// segment; row tiles are double-buffered by cp.async. Shared rows are
// row-major with a stride of dp + 4 floats (dp a multiple of 8), so the
// 16-byte loads of 16 threads reading 16 consecutive rows hit distinct banks.
//
// The scan keeps (score, row) when score <= the query's bound, the k-th
// smallest pivot-tile minimum times rho (see simt_rho); knn_select then
// re-scores the survivors in the reference's arithmetic order. L-inf scores
// are exact (a maximum does not depend on order, and |q - x| is rounded the
// same way), so its rho is 1.
//
// Replaces the L1 / L-inf / Hellinger branches of
// knn_compute_distance_matrix, crates/vector-cuda/src/kernels/knn.cu:21-201.
#include <algorithm>

#include "vrs_exact.cuh"
#include "vrs_internal.cuh"
#include "vrs_select.cuh"
#include "vrs_simt.cuh"

namespace vrs {
namespace simt {
namespace {

constexpr int SQ = 128;        // queries per CTA
constexpr int SN = 128;        // rows per tile
constexpr int THREADS = 256;   // 16 x 16; thread (ty, tx) owns queries ty + 16i, rows tx + 16j
constexpr int TQ = 8, TN = 8;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  // Zero-fills the 16 bytes when !valid (src-size 0).
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct SimtArgs {
  const float* base;  // row i of the scanned set is base[i * stride][0..dp)
  int64_t n;          // rows in the scanned set
  int64_t stride;     // 1 for the shard, s for the pivot set (every s-th row)
  int dp;
  const float* q;     // [nq][dp]
  int nq;
  int64_t seg_len;    // multiple of SN
  Cand* cand;         // [nseg][nq][cap]
  int* cnt;           // [nseg][nq]
  int* overflow;      // [nq]
  int cap;
  const float* init_bound;  // [nq] (append pass)
  float* tmin;              // [nq][tmin_stride] (pivot pass)
  int64_t tmin_stride;
};

// Loads rows [r0, r0 + SN) of the scanned set (base rows r * stride) into
// shared [SN][dp + 4]; rows at or past `rows` are zero-filled.
__device__ __forceinline__ void load_tile(float* dst, const float* src, int64_t r0, int64_t rows,
                                          int64_t stride, int dp) {
  const int ss = dp + 4;
  const int per_row = dp / 4;
  for (int i = threadIdx.x; i < SN * per_row; i += THREADS) {
    const int r = i / per_row, c = (i - r * per_row) * 4;
    const bool ok = r0 + r < rows;
    const float* g = src + (ok ? (r0 + r) * stride * dp + c : 0);
    cp_async16(dst + r * ss + c, g, ok);
  }
}

template <int METRIC>
__device__ __forceinline__ void accumulate(float (&acc)[TQ][TN], const float4 (&qv)[TQ], const float4 (&xv)[TN]) {
#pragma unroll
  for (int i = 0; i < TQ; i++) {
#pragma unroll
    for (int j = 0; j < TN; j++) {
      const float d0 = qv[i].x - xv[j].x, d1 = qv[i].y - xv[j].y;
      const float d2 = qv[i].z - xv[j].z, d3 = qv[i].w - xv[j].w;
      if (METRIC == vrs_exact::kL1) {
        acc[i][j] += fabsf(d0);
        acc[i][j] += fabsf(d1);
        acc[i][j] += fabsf(d2);
        acc[i][j] += fabsf(d3);
      } else if (METRIC == vrs_exact::kCheb) {
        acc[i][j] = fmaxf(acc[i][j], fabsf(d0));
        acc[i][j] = fmaxf(acc[i][j], fabsf(d1));
        acc[i][j] = fmaxf(acc[i][j], fabsf(d2));
        acc[i][j] = fmaxf(acc[i][j], fabsf(d3));
      } else {  // Hellinger: squared differences of the roots
        acc[i][j] = fmaf(d0, d0, acc[i][j]);
        acc[i][j] = fmaf(d1, d1, acc[i][j]);
        acc[i][j] = fmaf(d2, d2, acc[i][j]);
        acc[i][j] = fmaf(d3, d3, acc[i][j]);
      }
    }
  }
}

template <int METRIC, bool TILEMIN>
__global__ void __launch_bounds__(THREADS, 1) knn_scan_simt_kernel(SimtArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int ss = a.dp + 4;
  float* Qs = smem;                 // [SQ][ss]
  float* Xs = smem + SQ * ss;       // [2][SN][ss]
  int* s_cnt = reinterpret_cast<int*>(Xs + 2 * SN * ss);  // [SQ]
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int q0 = blockIdx.x * SQ;
  const int seg = blockIdx.y;
  const int64_t row_begin = (int64_t)seg * a.seg_len;
  const int64_t row_end = min(a.n, row_begin + a.seg_len);
  const int ntiles = row_end > row_begin ? (int)((row_end - row_begin + SN - 1) / SN) : 0;

  if (threadIdx.x < SQ) s_cnt[threadIdx.x] = 0;
  // Queries (zero rows past nq) and the first row tile.
  {
    const int per_row = a.dp / 4;
    for (int i = threadIdx.x; i < SQ * per_row; i += THREADS) {
      const int r = i / per_row, c = (i - r * per_row) * 4;
      const bool ok = q0 + r < a.nq;
      cp_async16(Qs + r * ss + c, a.q + (ok ? (int64_t)(q0 + r) * a.dp + c : 0), ok);
    }
  }
  if (ntiles > 0) load_tile(Xs, a.base, row_begin, row_end, a.stride, a.dp);
  cp_async_commit();

  float bound[TQ];
#pragma unroll
  for (int i = 0; i < TQ; i++) {
    const int q = q0 + ty + 16 * i;
    bound[i] = (!TILEMIN && q < a.nq && a.init_bound) ? a.init_bound[q] : -INFINITY;
  }

  for (int t = 0; t < ntiles; t++) {
    const int b = t & 1;
    if (t + 1 < ntiles)
      load_tile(Xs + (b ^ 1) * SN * ss, a.base, row_begin + (int64_t)(t + 1) * SN, row_end, a.stride, a.dp);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const float* xs = Xs + b * SN * ss;
    float acc[TQ][TN];
#pragma unroll
    for (int i = 0; i < TQ; i++)
#pragma unroll
      for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;
#pragma unroll 2
    for (int k = 0; k < a.dp; k += 4) {
      float4 qv[TQ], xv[TN];
#pragma unroll
      for (int i = 0; i < TQ; i++) qv[i] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * i) * ss + k);
#pragma unroll
      for (int j = 0; j < TN; j++) xv[j] = *reinterpret_cast<const float4*>(xs + (tx + 16 * j) * ss + k);
      accumulate<METRIC>(acc, qv, xv);
    }
    const int64_t r0 = row_begin + (int64_t)t * SN;
    if (TILEMIN) {
      // Tile minimum per query over the valid rows; the 16 threads of a
      // query row (one half-warp) combine by shuffles.
#pragma unroll
      for (int i = 0; i < TQ; i++) {
        float m = INFINITY;
#pragma unroll
        for (int j = 0; j < TN; j++)
          if (r0 + tx + 16 * j < row_end) m = fminf(m, acc[i][j]);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fminf(m, __shfl_xor_sync(0xffffffffu, m, o, 16));
        const int q = q0 + ty + 16 * i;
        if (tx == 0 && q < a.nq) a.tmin[(int64_t)q * a.tmin_stride + r0 / SN] = m;
      }
    } else {
#pragma unroll
      for (int i = 0; i < TQ; i++) {
        const int ql = ty + 16 * i;
#pragma unroll
        for (int j = 0; j < TN; j++) {
          const int64_t row = r0 + tx + 16 * j;
          if (acc[i][j] <= bound[i] && row < row_end) {
            const int pos = atomicAdd(&s_cnt[ql], 1);
            if (pos < a.cap)
              a.cand[((int64_t)seg * a.nq + q0 + ql) * a.cap + pos] = Cand{acc[i][j], (uint32_t)row};
          }
        }
      }
    }
    __syncthreads();  // the buffer just read is the next prefetch target
  }
  cp_async_wait<0>();
  if (!TILEMIN) {
    __syncthreads();
    if (threadIdx.x < SQ) {
      const int q = q0 + threadIdx.x;
      if (q < a.nq) {
        const int c = s_cnt[threadIdx.x];
        a.cnt[(int64_t)seg * a.nq + q] = min(c, a.cap);
        if (c > a.cap) a.overflow[q] = 1;
      }
    }
  }
}

// Starting bound per query: the k-th smallest pivot-tile minimum (each the
// score of a distinct pivot row) times rho.
__global__ void __launch_bounds__(256) simt_tau_kernel(const float* __restrict__ tmin, int ntile, int k,
                                                       float rho, float* __restrict__ init_bound) {
  extern __shared__ Cand buf[];
  __shared__ int s_hist[256];
  __shared__ int s_res[4];
  const int q = blockIdx.x;
  if (ntile < k) {
    if (threadIdx.x == 0) init_bound[q] = INFINITY;
    return;
  }
  const float* row = tmin + (int64_t)q * ntile;
  for (int t = threadIdx.x; t < ntile; t += blockDim.x) buf[t] = Cand{row[t], 0u};
  __syncthreads();
  const uint32_t kth = sel::block_select(buf, ntile, k, s_hist, s_res);
  if (threadIdx.x == 0) {
    const float tau = ord_inv(kth);
    init_bound[q] = isfinite(tau) ? __fmul_ru(tau, rho) : INFINITY;
  }
}

size_t smem_bytes(int dp) { return (size_t)(SQ + 2 * SN) * (dp + 4) * sizeof(float) + SQ * sizeof(int); }

template <int METRIC, bool TILEMIN>
int launch_one(const SimtArgs& a, int qtiles, int nseg, cudaStream_t s) {
  const size_t smem = smem_bytes(a.dp);
  VRS_CUDA(cudaFuncSetAttribute(knn_scan_simt_kernel<METRIC, TILEMIN>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  knn_scan_simt_kernel<METRIC, TILEMIN><<<dim3(qtiles, nseg), THREADS, smem, s>>>(a);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

template <bool TILEMIN>
int launch_metric(int metric, const SimtArgs& a, int qtiles, int nseg, cudaStream_t s) {
  switch (metric) {
    case vrs_exact::kL1: return launch_one<vrs_exact::kL1, TILEMIN>(a, qtiles, nseg, s);
    case vrs_exact::kCheb: return launch_one<vrs_exact::kCheb, TILEMIN>(a, qtiles, nseg, s);
    case vrs_exact::kHell: return launch_one<vrs_exact::kHell, TILEMIN>(a, qtiles, nseg, s);
  }
  set_error(VRS_ERR_INVALID_CONFIG, "CUDA-core scan: unsupported metric");
  return VRS_ERR_INVALID_CONFIG;
}

}  // namespace

bool simt_supported(int metric, int dp) {
  return (metric == vrs_exact::kL1 || metric == vrs_exact::kCheb || metric == vrs_exact::kHell) && dp % 8 == 0 &&
         dp <= kSimtMaxDp && smem_bytes(dp) <= 227 * 1024;
}

float simt_rho(int metric, int d) {
  if (metric == vrs_exact::kCheb) return 1.0f;
  // Sums of d non-negative terms in two orders differ from the exact sum of
  // the same terms by at most gamma_d = d u / (1 - d u) each; the bound
  // chains (approx -> exact -> k-th exact -> pivot approx) give
  // ((1 + g) / (1 - g))^2 < 1 + 5 g for small g; rounded up with slack.
  const double g = (double)(d + 2) * 0x1p-24;
  return (float)(1.0 + 5.0 * g) * (1.0f + 0x1p-20f);
}

SimtPlan simt_plan(int64_t n, int nq, int num_sms) {
  SimtPlan p;
  p.qtiles = (nq + SQ - 1) / SQ;
  const int64_t ntile = std::max<int64_t>(1, (n + SN - 1) / SN);
  // Segments: enough CTAs for ~8 waves of one CTA per SM, each segment at
  // least 4 tiles.
  int best = 1;
  double best_cost = 1e30;
  for (int nseg = 1; nseg <= 64; nseg++) {
    const int64_t tiles_per = (ntile + nseg - 1) / nseg;
    if (nseg > 1 && tiles_per < 4) break;
    const int64_t ctas = (int64_t)p.qtiles * nseg;
    const int64_t waves = (ctas + num_sms - 1) / num_sms;
    const double cost = (double)waves * tiles_per + 0.5 * nseg;  // wave-quantised time + per-CTA set-up
    if (cost < best_cost) {
      best_cost = cost;
      best = nseg;
    }
  }
  const int64_t tiles_per = (ntile + best - 1) / best;
  p.seg_len = tiles_per * SN;
  p.nseg = (int)std::max<int64_t>(1, (n + p.seg_len - 1) / p.seg_len);
  return p;
}

int simt_scan(const float* base, int64_t n, int64_t stride, int dp, const float* q, int nq, int metric,
              const SimtPlan& p, Cand* cand, int* cnt, int* overflow, int cap, const float* init_bound, float* tmin,
              int64_t tmin_stride, cudaStream_t s) {
  if (n == 0 || nq == 0) return VRS_OK;
  SimtArgs a;
  a.base = base;
  a.n = n;
  a.stride = stride;
  a.dp = dp;
  a.q = q;
  a.nq = nq;
  a.seg_len = p.seg_len;
  a.cand = cand;
  a.cnt = cnt;
  a.overflow = overflow;
  a.cap = cap;
  a.init_bound = init_bound;
  a.tmin = tmin;
  a.tmin_stride = tmin_stride;
  if (tmin) return launch_metric<true>(metric, a, p.qtiles, p.nseg, s);
  return launch_metric<false>(metric, a, p.qtiles, p.nseg, s);
}

int simt_tau(const float* tmin, int ntile, int nq, int k, float rho, float* init_bound, cudaStream_t s) {
  if (nq == 0) return VRS_OK;
  const size_t smem = (size_t)std::max(ntile, 1) * sizeof(Cand);
  if (smem > 200 * 1024) {
    set_error(VRS_ERR_INVALID_CONFIG, "pivot tile count too large");
    return VRS_ERR_INVALID_CONFIG;
  }
  VRS_CUDA(cudaFuncSetAttribute(simt_tau_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  simt_tau_kernel<<<nq, 256, smem, s>>>(tmin, ntile, k, rho, init_bound);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int64_t simt_tile_rows() { return SN; }

int64_t simt_pivot_rows(int64_t n, int k, int parts, int64_t* stride) {
  // About k * n / 256 rows (a few hundred candidates per query after the
  // bound), at most n / 6, and at least 32 tiles per k (a stable k-th tile
  // minimum); pooled over `parts` shards.
  int64_t m = n * std::max(k, 1) / 256;
  if (m > n / 6) m = n / 6;
  const int64_t lo = ((int64_t)32 * SN * std::max(k, 1) + parts - 1) / parts;
  if (m < lo) m = lo;
  if (m >= n) {
    *stride = 1;
    return n;
  }
  *stride = n / m;
  return n / *stride;
}

}  // namespace simt
}  // namespace vrs
