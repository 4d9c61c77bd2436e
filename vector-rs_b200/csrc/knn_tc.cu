// knn_tc.cu -- tensor-core (tcgen05) fused distance + candidate scan for the
// GEMM-form metrics (squared L2, Mahalanobis = sqrt L2, dot, cosine).
//
// Each CTA owns 256 queries (two M=128 fp16 operand tiles, loaded once by
// TMA) and streams 128-row fp16 tiles of one base segment through a 4-stage
// TMA ring. One thread issues tcgen05.mma into two 128x128 f32 accumulators
// per tile, double-buffered in TMEM (4 x 128 = 512 columns). Sixteen
// epilogue warps (one per TMEM lane quadrant, accumulator and column half)
// read their lanes with tcgen05.ld (one thread = one query), reduce each
// 64-column half to its best key, and only where that passes the query's
// acceptance bound append (score, row) to the query's segment list; lists
// are shrunk in place by a warp radix select when nearly full. The Q x N
// score matrix never reaches HBM.
//
// Correctness: fp16 products carry a bounded error; a row can belong to the
// exact top-k only if its approximate score is within `absm[q]` of the k-th
// best approximate score, so every such row is kept and later re-ranked in
// the reference's exact f32 arithmetic (knn_select in knn_kernels.cu).
//
// Replaces knn_compute_distance_matrix + knn_topk_select,
// crates/vector-cuda/src/kernels/knn.cu:21-305.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "tc_common.cuh"
#include "vrs_exact.cuh"
#include "vrs_exact_lanes.cuh"
#include "vrs_internal.cuh"
#include "vrs_select.cuh"
#include "vrs_tc.cuh"

namespace vrs {
namespace tc {
namespace {

constexpr int BM = 128;        // queries per accumulator
constexpr int NACC = 2;        // accumulators per CTA (256 queries)
constexpr int BN = 128;        // base rows per tile
constexpr int KBW = 64;        // 16-bit elements per K-block (one 128-byte swizzle row)
constexpr int MAX_KBLK = 2;    // D <= 128 on this path
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 16;   // 2 per (TMEM lane quadrant, accumulator): column halves
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr int HALF_COLS = BN / 2;
constexpr uint32_t BLK_A = BM * 128;  // bytes of one K-block of a 128-row tile
constexpr uint32_t BLK_B = BN * 128;
constexpr size_t SMEM_A = (size_t)NACC * MAX_KBLK * BLK_A;
constexpr size_t SMEM_B = (size_t)STAGES * MAX_KBLK * BLK_B;
constexpr size_t SMEM_HIST = (size_t)EPI_WARPS * 256 * 4;
constexpr size_t SMEM_BAR = 256;
constexpr size_t SMEM_TOTAL = 1024 + SMEM_A + SMEM_B + SMEM_HIST + SMEM_BAR;
constexpr uint64_t WAIT_NS = 2000000000ull;  // 2 s per wait, then abort
constexpr uint32_t TMEM_COLS = 512;
constexpr int kTauCap = 24576;  // pivot minima per query held in shared memory (192 KB)

struct TcScanArgs {
  const float* xn;   // |x|^2 per row (L2 mode), zero padded to a multiple of BN
  int64_t n;
  int nq;
  int ksteps;        // ceil(D / 16)
  int kblk;          // ceil(D16 / 64)
  int64_t seg_len;   // multiple of BN
  Cand* cand;        // [nseg * 2][nq][cap]: one list per (segment, column half, query)
  int* cnt;          // [nseg * 2][nq]
  int* overflow;     // [nq]
  int cap;
  int k;
  const float* absm; // [nq]
  int* err;          // global error word (0 = ok)
  // Pivot pass: instead of appending, write the minimum score of each
  // column part of every group of kPivotGroup tiles per query to
  // tmin[query][parts * group + part] (one-SM kernel: 128-row tiles, two
  // 64-column halves; pair kernel: 256-row tiles, four 64-column quarters;
  // group = global tile / kPivotGroup; segments start on group boundaries).
  // Every value is the minimum over 256 distinct rows.
  float* tmin;
  int64_t tmin_stride;  // entries per query row of tmin (parts * groups)
  // Starting acceptance bound per query (null: +inf).
  const float* init_bound;
  uint32_t idesc;    // MMA instruction descriptor
  // Operand scales (powers of two): accumulators are qscale[q] * xscale
  // times the unscaled products.
  const float* qscale;
  float xscale;
};

// MODE 0: heap score = |x|^2 - 2 acc (squared L2, Mahalanobis);
// MODE 1: heap score = -acc (dot, cosine on unit rows);
// MODE 2: heap score = -2 acc, where the operands carry -|x|^2 / 2 in two
//         extra K columns (squared L2 and Mahalanobis with d <= 126).
// The epilogue works on a per-mode "key" whose best end is the minimum
// (MODE 0: the score) or the maximum (MODE 1 and 2: acc). TILEMIN selects
// the pivot pass.
template <int MODE, bool TILEMIN>
__global__ void __launch_bounds__(THREADS, 1)
    knn_scan_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       TcScanArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + SMEM_A;
  int* s_hist = (int*)(sB + SMEM_B);
  uint64_t* bars = (uint64_t*)((uint8_t*)s_hist + SMEM_HIST);
  uint64_t* full = bars;                // [STAGES] TMA -> MMA
  uint64_t* empty = bars + STAGES;      // [STAGES] MMA -> TMA
  uint64_t* tfull = bars + 2 * STAGES;  // [2] MMA -> epilogue
  uint64_t* tempty = tfull + 2;         // [2] epilogue -> MMA
  uint64_t* afull = tempty + 2;         // queries loaded
  uint32_t* s_tmem = (uint32_t*)(afull + 1);
  volatile int* s_abort = (volatile int*)(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * (BM * NACC);
  const int seg = blockIdx.y;
  const int64_t row_begin = (int64_t)seg * a.seg_len;
  const int64_t row_end = min(a.n, row_begin + a.seg_len);
  const int ntiles = row_end > row_begin ? (int)((row_end - row_begin + BN - 1) / BN) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    mbar_init(afull, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc(s_tmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---------------------------------------------------- TMA producer
    if (lane == 0 && ntiles > 0) {
      mbar_expect_tx(afull, (uint32_t)(NACC * a.kblk) * BLK_A);
      for (int acc = 0; acc < NACC; acc++)
        for (int kb = 0; kb < a.kblk; kb++)
          tma_load_2d(sA + (acc * MAX_KBLK + kb) * BLK_A, &tmA, kb * KBW, q0 + acc * BM, afull);
      int issued = 0;
      for (int t = 0; t < ntiles; t++) {
        const int s = t % STAGES;
        if (!mbar_wait(&empty[s], ((t / STAGES) & 1) ^ 1, s_abort, a.err, 1, WAIT_NS)) break;
        mbar_expect_tx(&full[s], (uint32_t)a.kblk * BLK_B);
        const int y = (int)(row_begin + (int64_t)t * BN);
        for (int kb = 0; kb < a.kblk; kb++)
          tma_load_2d(sB + (s * MAX_KBLK + kb) * BLK_B, &tmB, kb * KBW, y, &full[s]);
        issued = t + 1;
      }
      if (*s_abort) {
        // Drain: wait (bounded) for the loads this thread issued.
        volatile int dummy = 0;
        for (int t = max(0, issued - STAGES); t < issued; t++)
          mbar_wait(&full[t % STAGES], (t / STAGES) & 1, &dummy, a.err, 0, WAIT_NS / 4);
        mbar_wait(afull, 0, &dummy, a.err, 0, WAIT_NS / 4);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc = a.idesc;
      // This thread shares its scheduler with four epilogue warps, so each
      // MMA should cost it about one instruction: the A descriptors (fixed
      // for the CTA) are formed once into registers, the B descriptors once
      // per tile. Descriptors differ only in the masked start-address field.
      const DescSw128 a_desc(sA), b_desc(sB);
      const int ksteps = a.ksteps;
      uint64_t ad[NACC][MAX_KBLK * 4];
#pragma unroll
      for (int acc = 0; acc < NACC; acc++)
#pragma unroll
        for (int ks = 0; ks < MAX_KBLK * 4; ks++)
          ad[acc][ks] = a_desc.at((uint32_t)(acc * MAX_KBLK * BLK_A + (ks >> 2) * BLK_A + (ks & 3) * 32) >> 4);
      bool ok = mbar_wait(afull, 0, s_abort, a.err, 2, WAIT_NS);
      tc_fence_after();
      int last = -1;
      for (int t = 0; ok && t < ntiles; t++) {
        const int s = t % STAGES, b = t & 1;
        uint64_t bd[MAX_KBLK * 4];
#pragma unroll
        for (int ks = 0; ks < MAX_KBLK * 4; ks++)
          bd[ks] = b_desc.at((uint32_t)(s * MAX_KBLK * BLK_B + (ks >> 2) * BLK_B + (ks & 3) * 32) >> 4);
        if (!mbar_wait(&full[s], (t / STAGES) & 1, s_abort, a.err, 3, WAIT_NS)) break;
        if (!mbar_wait(&tempty[b], ((t >> 1) & 1) ^ 1, s_abort, a.err, 4, WAIT_NS)) break;
        tc_fence_after();
#pragma unroll
        for (int acc = 0; acc < NACC; acc++) {
          const uint32_t d = tmem + acc * 256 + b * BN;
#pragma unroll
          for (int ks = 0; ks < MAX_KBLK * 4; ks++)
            if (ks < ksteps) mma_f16(d, ad[acc][ks], bd[ks], idesc, ks > 0 ? 1u : 0u);
        }
        mma_commit(&empty[s]);
        mma_commit(&tfull[b]);
        last = t;
      }
      if (*s_abort && last >= 0) {
        // Let the last issued MMAs finish before TMEM is released.
        volatile int dummy = 0;
        mbar_wait(&tfull[last & 1], (last >> 1) & 1, &dummy, a.err, 0, WAIT_NS / 4);
      }
    }
  } else {
    // ---------------------------------------------------- epilogue
    // Warp e owns TMEM lane quadrant (warp % 4) of accumulator (e / 4) % 2
    // and column half e / 8 of every tile: one thread = one query.
    const int ew = warp - 2;
    const int acc = (ew >> 2) & 1;
    const int ch = ew >> 3;
    const int quad = warp & 3;
    const int q = q0 + acc * BM + quad * 32 + lane;
    const bool vq = q < a.nq;
    const int64_t list_id = ((int64_t)blockIdx.y * 2 + ch) * a.nq + (vq ? q : 0);
    Cand* list = a.cand + list_id * a.cap;
    int count = 0;
    // Acceptance bound on the heap score; -inf for padding queries, so that
    // nothing passes for them.
    float bound = vq ? (a.init_bound ? a.init_bound[q] : INFINITY) : -INFINITY;
    // Accumulator scale of this query and its inverse (both exact powers of two).
    const float ks = vq ? a.qscale[q] * a.xscale : 1.0f;
    const float inv_ks = 1.0f / ks;
    const float f2 = -2.0f * inv_ks;
    const float absm = vq ? a.absm[q] : 0.0f;
    int* hist = s_hist + ew * 256;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    float run = MODE == 0 ? INFINITY : -INFINITY;  // pivot pass: best key of the current group
    for (int t = 0; t < ntiles; t++) {
      const int b = t & 1;
      const bool ok = mbar_wait(&tfull[b], (t >> 1) & 1, s_abort, a.err, 5, WAIT_NS);
      if (!__all_sync(sel::kFull, ok)) break;
      tc_fence_after();
      const int64_t n0 = row_begin + (int64_t)t * BN + ch * HALF_COLS;
      if (MODE == 0 && t + 1 < ntiles && lane < 2) {
        // |x|^2 of this warp's columns of the next tile -> L1 (2 lines).
        asm volatile("prefetch.global.L1 [%0];" ::"l"(a.xn + n0 + BN + lane * 32));
      }
      const int64_t rem_cols = row_end - n0;
      const int valid_cols = rem_cols < HALF_COLS ? (int)(rem_cols > 0 ? rem_cols : 0) : HALF_COLS;
      // Key threshold: MODE 0 passes key <= bound, MODE 1 key >= -bound ks,
      // MODE 2 key >= -bound ks / 2 (all factors are exact powers of two).
      const float thr = MODE == 0 ? bound : MODE == 1 ? -bound * ks : -0.5f * bound * ks;
      // The warp's whole column half: 64 accumulators per thread, one wait.
      float v[HALF_COLS];
      tmem_ld64(tmem + lane_base + acc * 256 + b * BN + ch * HALF_COLS, v);
      // The tile's columns are in registers: hand the TMEM buffer back to
      // the MMA issuer now, so the selection below overlaps the next MMAs.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      if (MODE == 0) {
        const float4* xp = reinterpret_cast<const float4*>(a.xn + n0);
#pragma unroll
        for (int j4 = 0; j4 < HALF_COLS / 4; j4++) {
          // Four loads in flight at a time keep the register count under
          // the 96 that 18 warps per SM allow.
          if (j4 % 4 == 0) asm volatile("" ::: "memory");
          const float4 x4 = __ldg(xp + j4);
          v[4 * j4 + 0] = fmaf(f2, v[4 * j4 + 0], x4.x);
          v[4 * j4 + 1] = fmaf(f2, v[4 * j4 + 1], x4.y);
          v[4 * j4 + 2] = fmaf(f2, v[4 * j4 + 2], x4.z);
          v[4 * j4 + 3] = fmaf(f2, v[4 * j4 + 3], x4.w);
        }
      }
      if (valid_cols < HALF_COLS) {
        // Columns past the segment end (the segment's last tile only): the
        // worst key for the pivot minima; NaN for the append path, which
        // fails every comparison (min/max ignore a NaN operand) even when
        // the bound is infinite.
        const float pad = TILEMIN ? (MODE == 0 ? INFINITY : -INFINITY) : __int_as_float(0x7fffffff);
#pragma unroll
        for (int j = 0; j < HALF_COLS; j++)
          if (j >= valid_cols) v[j] = pad;
      }
      // Best key of each group of 8 columns, then of the half: 36 three-input
      // min/max for 64 keys. The per-group tests run only in lanes whose
      // half passes.
      float g[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float* w = v + 8 * i;
        g[i] = MODE == 0 ? fmin3(fmin3(w[0], w[1], w[2]), fmin3(w[3], w[4], w[5]), fminf(w[6], w[7]))
                         : fmax3(fmax3(w[0], w[1], w[2]), fmax3(w[3], w[4], w[5]), fmaxf(w[6], w[7]));
      }
      const float best = MODE == 0 ? fmin3(fmin3(g[0], g[1], g[2]), fmin3(g[3], g[4], g[5]), fminf(g[6], g[7]))
                                   : fmax3(fmax3(g[0], g[1], g[2]), fmax3(g[3], g[4], g[5]), fmaxf(g[6], g[7]));
      if (!TILEMIN && (MODE == 0 ? best <= thr : best >= thr)) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
          if (MODE == 0 ? g[i] <= thr : g[i] >= thr) {
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
              const float sc = MODE == 0 ? v[8 * i + jj] : MODE == 1 ? -inv_ks * v[8 * i + jj] : f2 * v[8 * i + jj];
              if (sc <= bound) list[count++] = Cand{sc, (uint32_t)(n0 + 8 * i + jj)};
            }
          }
        }
      }
      if (TILEMIN) {
        run = MODE == 0 ? fminf(run, best) : fmaxf(run, best);
        if ((t + 1) % kPivotGroup == 0 || t == ntiles - 1) {
          if (vq)
            a.tmin[(int64_t)q * a.tmin_stride + (row_begin / BN + t) / kPivotGroup * 2 + ch] =
                MODE == 0 ? run : MODE == 1 ? -inv_ks * run : f2 * run;
          run = MODE == 0 ? INFINITY : -INFINITY;
        }
        continue;
      }
      // Shrink lists that could overflow on the next tile.
      unsigned need = __ballot_sync(sel::kFull, vq && count > a.cap - HALF_COLS);
      while (need) {
        const int l = __ffs(need) - 1;
        need &= need - 1;
        const int lc = __shfl_sync(sel::kFull, count, l);
        const float la = __shfl_sync(sel::kFull, absm, l);
        Cand* ll = reinterpret_cast<Cand*>(
            __shfl_sync(sel::kFull, reinterpret_cast<unsigned long long>(list), l));
        __syncwarp();
        int less;
        const uint32_t kth = sel::warp_select<false>(ll, lc, a.k, 0, hist, &less);
        const float bnd = __fadd_ru(ord_inv(kth), la);
        const int nc = sel::warp_filter(ll, lc, sel::KeepBound{bnd});
        if (lane == l) {
          count = nc;
          bound = bnd;
          if (nc > a.cap - HALF_COLS) {
            a.overflow[q] = 1;
            count = 0;
            bound = -INFINITY;
          }
        }
      }
    }
    if (vq && !TILEMIN) a.cnt[list_id] = count;
    if (vq && *s_abort) a.overflow[q] = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------- 2-SM scan (cta_group::2)
// The candidate pass, and with TILEMIN the pivot pass, on CTA pairs
// (N = 256 by default; KNN_P_BN = 128 builds a 128-row pair tile with four
// accumulator buffers, measured slower on C2). A cluster of two CTAs on two SMs owns 256
// queries (128 per CTA, its A tile) and streams 256-row base tiles, each CTA
// loading its 128-row half. The even CTA's one thread issues
// tcgen05.mma.cta_group::2 with M = 256, N = 256: every CTA's TMEM receives
// its 128 queries x the tile's 256 rows, double-buffered (2 x 256 = 512
// columns). Per SM and MMA the operands read from shared memory halve
// against the 1-SM M = 128 x N = 128 tile (one A and one half-B K-slice for
// twice the products).
//   * TMA: both CTAs' loads complete on the even CTA's `full` / `afull`
//     barriers (armed by the even CTA with both halves' bytes); a stage is
//     refilled after the MMA commit arrives on that CTA's own `empty`
//     (multicast to both CTAs).
//   * The MMA commit also arrives on both CTAs' `tfull`; each CTA's 16
//     epilogue warps (TMEM lane quadrant x 64-column quarter: one thread =
//     one query, 64 columns per tile, the epilogue of the 1-SM kernel) load
//     their columns and at once arrive on the even CTA's `tempty`, then test
//     and append.
//   * Lists: one per (segment, column quarter, query); the pivot pass
//     writes one minimum per (query, quarter, group of kPivotGroup tiles).
// Every wait is bounded; both CTAs meet in a cluster barrier before TMEM
// is released and before either exits.
#ifndef KNN_P_BN
#define KNN_P_BN 256
#endif
constexpr int P_BM = 128;             // queries per CTA (M = 256 per pair)
constexpr int P_BN = KNN_P_BN;        // base rows per pair tile (N)
constexpr int P_HALF = P_BN / 2;      // rows each CTA loads
constexpr int P_NBUF = 512 / P_BN;    // accumulator buffers in TMEM
constexpr int P_QUARTER = P_BN / 4;   // columns per epilogue warp
constexpr uint32_t P_BLK = 128 * 128;        // bytes of one K-block of the 128-row A tile
constexpr uint32_t P_BLK_B = P_HALF * 128;   // bytes of one K-block of a CTA's B half
constexpr int P_STAGES = (int)((160u * 1024u) / (MAX_KBLK * P_BLK_B));
constexpr size_t P_SMEM_BAR = 512;
constexpr size_t P_SMEM_A = (size_t)MAX_KBLK * P_BLK;
constexpr size_t P_SMEM_B = (size_t)P_STAGES * MAX_KBLK * P_BLK_B;
constexpr size_t P_SMEM_TOTAL = 1024 + P_SMEM_A + P_SMEM_B + SMEM_HIST + P_SMEM_BAR;
static_assert(P_BN == 128 || P_BN == 256, "2-SM scan: pair tiles are 128 or 256 rows");
static_assert(P_QUARTER % 32 == 0, "2-SM scan: epilogue columns come in 32-column loads");
static_assert(P_SMEM_TOTAL <= 232448, "2-SM scan: shared memory above the per-block limit");
static_assert((2 * P_STAGES + 2 * P_NBUF + 1) * 8 + 8 <= P_SMEM_BAR, "2-SM scan: barrier region too small");

template <int MODE, bool TILEMIN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    knn_scan_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        TcScanArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_SMEM_A;
  int* s_hist = (int*)(sB + P_SMEM_B);
  uint64_t* bars = (uint64_t*)((uint8_t*)s_hist + SMEM_HIST);
  uint64_t* full = bars;                  // [P_STAGES] even CTA: both halves' bytes
  uint64_t* empty = bars + P_STAGES;      // [P_STAGES] each CTA: MMA commit
  uint64_t* tfull = bars + 2 * P_STAGES;  // [P_NBUF] each CTA: MMA commit
  uint64_t* tempty = tfull + P_NBUF;      // [P_NBUF] even CTA: both CTAs' epilogue warps
  uint64_t* afull = tempty + P_NBUF;      // even CTA: both A tiles
  uint32_t* s_tmem = (uint32_t*)(afull + 1);
  volatile int* s_abort = (volatile int*)(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const bool lead = cta == 0;
  const int q0 = (blockIdx.x >> 1) * (2 * P_BM) + (int)cta * P_BM;
  const int seg = blockIdx.y;
  const int64_t row_begin = (int64_t)seg * a.seg_len;
  const int64_t row_end = min(a.n, row_begin + a.seg_len);
  const int ntiles = row_end > row_begin ? (int)((row_end - row_begin + P_BN - 1) / P_BN) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < P_NBUF; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EPI_WARPS);
    }
    mbar_init(afull, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(s_tmem, TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---------------------------------------------------- TMA producer
    if (lane == 0 && ntiles > 0) {
      const uint32_t afull_lead = mapa_shared(afull, 0);
      if (lead) mbar_expect_tx(afull, (uint32_t)(2 * a.kblk) * P_BLK);
      for (int kb = 0; kb < a.kblk; kb++) tma_load_2d_pair(sA + kb * P_BLK, &tmA, kb * KBW, q0, afull_lead);
      int issued = 0;
      for (int t = 0; t < ntiles; t++) {
        const int s = t % P_STAGES;
        if (!mbar_wait(&empty[s], ((t / P_STAGES) & 1) ^ 1, s_abort, a.err, 21, WAIT_NS)) break;
        if (lead) mbar_expect_tx(&full[s], (uint32_t)(2 * a.kblk) * P_BLK_B);
        const uint32_t full_lead = mapa_shared(&full[s], 0);
        const int y = (int)(row_begin + (int64_t)t * P_BN + (int)cta * P_HALF);
        for (int kb = 0; kb < a.kblk; kb++)
          tma_load_2d_pair(sB + (s * MAX_KBLK + kb) * P_BLK_B, &tmB, kb * KBW, y, full_lead);
        issued = t + 1;
      }
      if (*s_abort && lead) {
        // Drain (bounded): both CTAs' loads complete on these barriers.
        volatile int dummy = 0;
        for (int t = max(0, issued - P_STAGES); t < issued; t++)
          mbar_wait(&full[t % P_STAGES], (t / P_STAGES) & 1, &dummy, a.err, 0, WAIT_NS / 4);
        mbar_wait(afull, 0, &dummy, a.err, 0, WAIT_NS / 4);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer (even CTA)
    if (lane == 0 && lead && ntiles > 0) {
      const uint32_t idesc = a.idesc;
      const DescSw128 a_desc(sA), b_desc(sB);
      const int ksteps = a.ksteps;
      uint64_t ad[MAX_KBLK * 4];
#pragma unroll
      for (int ks = 0; ks < MAX_KBLK * 4; ks++) ad[ks] = a_desc.at((uint32_t)((ks >> 2) * P_BLK + (ks & 3) * 32) >> 4);
      bool ok = mbar_wait(afull, 0, s_abort, a.err, 22, WAIT_NS);
      tc_fence_after();
      int last = -1;
      for (int t = 0; ok && t < ntiles; t++) {
        const int s = t % P_STAGES, b = t % P_NBUF;
        uint64_t bd[MAX_KBLK * 4];
#pragma unroll
        for (int ks = 0; ks < MAX_KBLK * 4; ks++)
          bd[ks] = b_desc.at((uint32_t)(s * MAX_KBLK * P_BLK_B + (ks >> 2) * P_BLK_B + (ks & 3) * 32) >> 4);
        if (!mbar_wait(&full[s], (t / P_STAGES) & 1, s_abort, a.err, 23, WAIT_NS)) break;
        if (!mbar_wait(&tempty[b], ((t / P_NBUF) & 1) ^ 1, s_abort, a.err, 24, WAIT_NS)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * P_BN;
#pragma unroll
        for (int ks = 0; ks < MAX_KBLK * 4; ks++)
          if (ks < ksteps) mma_f16_pair(d, ad[ks], bd[ks], idesc, ks > 0 ? 1u : 0u);
        mma_commit_pair(&empty[s], 0x3);
        mma_commit_pair(&tfull[b], 0x3);
        last = t;
      }
      if (*s_abort && last >= 0) {
        volatile int dummy = 0;
        mbar_wait(&tfull[last % P_NBUF], (last / P_NBUF) & 1, &dummy, a.err, 0, WAIT_NS / 4);
      }
    }
  } else {
    // ---------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int quarter = ew >> 2;
    const int quad = warp & 3;
    const int q = q0 + quad * 32 + lane;
    const bool vq = q < a.nq;
    const int64_t list_id = ((int64_t)blockIdx.y * 4 + quarter) * a.nq + (vq ? q : 0);
    Cand* list = TILEMIN ? nullptr : a.cand + list_id * a.cap;
    int count = 0;
    float bound = vq ? (a.init_bound ? a.init_bound[q] : INFINITY) : -INFINITY;
    const float ks = vq ? a.qscale[q] * a.xscale : 1.0f;
    const float inv_ks = 1.0f / ks;
    const float f2 = -2.0f * inv_ks;
    const float absm = vq ? a.absm[q] : 0.0f;
    int* hist = s_hist + ew * 256;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    constexpr int NGR = P_QUARTER / 8;  // groups of 8 columns per warp and tile
    float run = MODE == 0 ? INFINITY : -INFINITY;  // pivot pass: best key of the current group
    for (int t = 0; t < ntiles; t++) {
      const int b = t % P_NBUF;
      const bool ok = mbar_wait(&tfull[b], (t / P_NBUF) & 1, s_abort, a.err, 25, WAIT_NS);
      if (!__all_sync(sel::kFull, ok)) break;
      tc_fence_after();
      const int64_t n0 = row_begin + (int64_t)t * P_BN + quarter * P_QUARTER;
      if (MODE == 0 && t + 1 < ntiles && lane < P_QUARTER / 32)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(a.xn + n0 + P_BN + lane * 32));
      const int64_t rem_cols = row_end - n0;
      const int valid_cols = rem_cols < P_QUARTER ? (int)(rem_cols > 0 ? rem_cols : 0) : P_QUARTER;
      const float thr = MODE == 0 ? bound : MODE == 1 ? -bound * ks : -0.5f * bound * ks;
      float v[P_QUARTER];
      if constexpr (P_QUARTER == 64)
        tmem_ld64(tmem + lane_base + b * P_BN + quarter * P_QUARTER, v);
      else
        tmem_ld32(tmem + lane_base + b * P_BN + quarter * P_QUARTER, v);
      // The tile's columns are in registers: hand the TMEM buffer back to
      // the MMA issuer now, so the selection below overlaps the next MMAs.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (lead)
          mbar_arrive(&tempty[b]);
        else
          mbar_arrive_cluster(mapa_shared(&tempty[b], 0));
      }
      if (MODE == 0) {
        const float4* xp = reinterpret_cast<const float4*>(a.xn + n0);
#pragma unroll
        for (int j4 = 0; j4 < P_QUARTER / 4; j4++) {
          if (j4 % 4 == 0) asm volatile("" ::: "memory");
          const float4 x4 = __ldg(xp + j4);
          v[4 * j4 + 0] = fmaf(f2, v[4 * j4 + 0], x4.x);
          v[4 * j4 + 1] = fmaf(f2, v[4 * j4 + 1], x4.y);
          v[4 * j4 + 2] = fmaf(f2, v[4 * j4 + 2], x4.z);
          v[4 * j4 + 3] = fmaf(f2, v[4 * j4 + 3], x4.w);
        }
      }
      if (valid_cols < P_QUARTER) {
        // Columns past the segment end: the worst key for the pivot minima;
        // NaN for the append path, which fails every comparison.
        const float pad = TILEMIN ? (MODE == 0 ? INFINITY : -INFINITY) : __int_as_float(0x7fffffff);
#pragma unroll
        for (int j = 0; j < P_QUARTER; j++)
          if (j >= valid_cols) v[j] = pad;
      }
      float g[NGR];
#pragma unroll
      for (int i = 0; i < NGR; i++) {
        const float* w = v + 8 * i;
        g[i] = MODE == 0 ? fmin3(fmin3(w[0], w[1], w[2]), fmin3(w[3], w[4], w[5]), fminf(w[6], w[7]))
                         : fmax3(fmax3(w[0], w[1], w[2]), fmax3(w[3], w[4], w[5]), fmaxf(w[6], w[7]));
      }
      float best;
      if constexpr (NGR == 8)
        best = MODE == 0 ? fmin3(fmin3(g[0], g[1], g[2]), fmin3(g[3], g[4], g[5]), fminf(g[6], g[7]))
                         : fmax3(fmax3(g[0], g[1], g[2]), fmax3(g[3], g[4], g[5]), fmaxf(g[6], g[7]));
      else
        best = MODE == 0 ? fminf(fmin3(g[0], g[1], g[2]), g[3]) : fmaxf(fmax3(g[0], g[1], g[2]), g[3]);
      if (TILEMIN) {
        run = MODE == 0 ? fminf(run, best) : fmaxf(run, best);
        if ((t + 1) % kPivotGroup == 0 || t == ntiles - 1) {
          if (vq)
            a.tmin[(int64_t)q * a.tmin_stride + (row_begin / P_BN + t) / kPivotGroup * 4 + quarter] =
                MODE == 0 ? run : MODE == 1 ? -inv_ks * run : f2 * run;
          run = MODE == 0 ? INFINITY : -INFINITY;
        }
        continue;
      }
      if (MODE == 0 ? best <= thr : best >= thr) {
#pragma unroll
        for (int i = 0; i < NGR; i++) {
          if (MODE == 0 ? g[i] <= thr : g[i] >= thr) {
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
              const float sc = MODE == 0 ? v[8 * i + jj] : MODE == 1 ? -inv_ks * v[8 * i + jj] : f2 * v[8 * i + jj];
              if (sc <= bound) list[count++] = Cand{sc, (uint32_t)(n0 + 8 * i + jj)};
            }
          }
        }
      }
      // Shrink lists that could overflow on the next tile.
      unsigned need = __ballot_sync(sel::kFull, vq && count > a.cap - P_QUARTER);
      while (need) {
        const int l = __ffs(need) - 1;
        need &= need - 1;
        const int lc = __shfl_sync(sel::kFull, count, l);
        const float la = __shfl_sync(sel::kFull, absm, l);
        Cand* ll = reinterpret_cast<Cand*>(
            __shfl_sync(sel::kFull, reinterpret_cast<unsigned long long>(list), l));
        __syncwarp();
        int less;
        const uint32_t kth = sel::warp_select<false>(ll, lc, a.k, 0, hist, &less);
        const float bnd = __fadd_ru(ord_inv(kth), la);
        const int nc = sel::warp_filter(ll, lc, sel::KeepBound{bnd});
        if (lane == l) {
          count = nc;
          bound = bnd;
          if (nc > a.cap - P_QUARTER) {
            a.overflow[q] = 1;
            count = 0;
            bound = -INFINITY;
          }
        }
      }
    }
    if (vq && !TILEMIN) a.cnt[list_id] = count;
    if (vq && *s_abort) a.overflow[q] = 1;
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no MMA, load or remote arrival of either CTA is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ prep
// Base rows -> fp16 operand rows (cosine: unit-normalised), |x|^2 for the L2
// epilogue, max |x| for the margins, and the list of near-zero cosine rows.
// One 2-byte tensor-core operand: fp16 for cosine, bf16 otherwise.
__device__ __forceinline__ uint16_t to_operand(float v, bool f16) {
  return f16 ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__global__ void tc_base_prep_kernel(const float* __restrict__ x, int64_t n, int d, int dp, int d16,
                                    int metric, float xscale, int fold_m, uint16_t* __restrict__ xb,
                                    float* __restrict__ xn, unsigned int* __restrict__ xmax_bits,
                                    uint32_t* __restrict__ tiny, int* __restrict__ n_tiny,
                                    int tiny_cap) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  const float* v = x + r * dp;
  uint16_t* o = xb + r * d16;
  const bool f16 = tc_fp16(metric);
  float scale = 1.0f;
  if (metric == vrs_exact::kCos) {
    const float sx = sqrtf(vrs_exact::cos_norm_sq(v, d));
    if (!(sx >= kTinyNorm)) {
      int i = atomicAdd(n_tiny, 1);
      if (i < tiny_cap) tiny[i] = (uint32_t)r;
      scale = 0.0f;
    } else {
      scale = 1.0f / sx;
    }
  }
  double ss = 0.0;
  for (int j = 0; j < d16; j++) {
    float e = j < d ? v[j] : 0.0f;
    ss += (double)e * (double)e;
    o[j] = to_operand(metric == vrs_exact::kCos ? e * scale : e * xscale, f16);
  }
  if (tc_fold(metric, d)) {
    // F = -xscale |x|^2 / 2^(fold_m + 1) as hi + lo fp16 in columns d and
    // d + 1 (|F| <= 2^14 by the choice of fold_m); queries put
    // qscale * 2^fold_m there, so the accumulator gains -qscale xscale |x|^2 / 2.
    const double t = -(double)xscale * ss * ldexp(1.0, -(fold_m + 1));
    const __half hi = __double2half(t);
    o[d] = __half_as_ushort(hi);
    o[d + 1] = __half_as_ushort(__double2half(t - (double)__half2float(hi)));
  }
  if (xn) xn[r] = (float)ss;
  atomicMax(xmax_bits, __float_as_uint((float)sqrt(ss)));
}

// Queries -> padded f32 rows for the exact re-rank (and, for cosine, their
// norms in the reference's order), fp16 operand rows, per-query operand
// scales and acceptance margins (heap-score units). One warp per query: lane
// l holds columns l, l + 32, l + 64, l + 96 (d <= 128 on this path). Near-zero
// cosine queries are routed to the exact fallback.
constexpr int kPrepWarps = 8;

__global__ void __launch_bounds__(kPrepWarps * 32)
    tc_query_prep_kernel(const float* __restrict__ q_in, int nq, int d, int dp, int d16, int metric,
                         const unsigned int* __restrict__ xmax_bits, float xscale, int fold_m,
                         float* __restrict__ qpad, float* __restrict__ qaux, uint16_t* __restrict__ qb,
                         float* __restrict__ qscale, float* __restrict__ absm, int* __restrict__ overflow,
                         float* __restrict__ qsq) {
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
  if (i >= nq) return;  // uniform per warp
  const float* src = q_in + (int64_t)i * d;
  float v[4];
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const int c = lane + 32 * t;
    v[t] = c < d ? src[c] : 0.0f;
    if (c < dp) qpad[(int64_t)i * dp + c] = v[t];
  }
  const bool f16 = tc_fp16(metric);
  float scale = 1.0f;
  if (metric == vrs_exact::kCos) {
    // cos_norm_sq in the reference's order (vrs_exact.cuh): lane l < 16
    // plays SIMD lane l of s0, lane l + 16 of s1; chunks of 32 in order,
    // then one 16-wide step, the halving tree, and the tail in order.
    const int chunks = d / 32;
    float acc = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; t++)
      if (t < chunks) acc = __fmaf_rn(v[t], v[t], acc);
    int e0 = chunks * 32;
    if (e0 + 16 <= d) {
      const float x = chunks == 0 ? v[0] : chunks == 1 ? v[1] : chunks == 2 ? v[2] : v[3];
      if (lane < 16) acc = __fmaf_rn(x, x, acc);
      e0 += 16;
    }
    const float s1 = __shfl_down_sync(0xffffffffu, acc, 16);
    float r = vrs_exact::lanes::hsum16(__fadd_rn(acc, s1));
    r = __shfl_sync(0xffffffffu, r, 0);
    for (int e = e0; e < d; e++) {  // uniform
      const int t = e >> 5;
      const float x = __shfl_sync(0xffffffffu, t == 0 ? v[0] : t == 1 ? v[1] : t == 2 ? v[2] : v[3], e & 31);
      r = __fadd_rn(r, __fmul_rn(x, x));
    }
    if (lane == 0 && qaux) qaux[i] = r;
    const float sq = sqrtf(r);
    if (!(sq >= kTinyNorm)) {
      if (lane == 0) overflow[i] = 1;
      scale = 0.0f;
    } else {
      scale = 1.0f / sq;
    }
  }
  // Query scale: largest element into [2^7, 2^8) (unit cosine rows: 1);
  // with the folded |x|^2 the fold column qs 2^fold_m must stay a normal
  // fp16 (<= 2^15, >= 2^-14); a query that cannot meet both goes to the
  // exact scan.
  const bool fold = tc_fold(metric, d);
  float qs = 1.0f;
  if (metric != vrs_exact::kCos) {
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int ex = mx > 0.0f ? 7 - ilogbf(mx) : 0;
    ex = max(-60, min(60, ex));
    if (fold) {
      ex = min(ex, 15 - fold_m);
      if ((ex < -14 - fold_m || (mx > 0.0f && ldexpf(mx, ex) > 32768.0f)) && lane == 0) overflow[i] = 1;
    }
    qs = ldexpf(1.0f, ex);
  }
  double ss = 0.0;
#pragma unroll
  for (int t = 0; t < 4; t++) ss += (double)v[t] * (double)v[t];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  uint16_t* o = qb + (int64_t)i * d16;
  const uint16_t fc = __half_as_ushort(__float2half_rn(ldexpf(qs, fold_m)));
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const int c = lane + 32 * t;
    if (c < d16) {
      uint16_t w = to_operand(metric == vrs_exact::kCos ? v[t] * scale : v[t] * qs, f16);
      if (fold && (c == d || c == d + 1)) w = fc;
      o[c] = w;
    }
  }
  if (lane != 0) return;
  qscale[i] = qs;
  // |q|^2 from below (the squares and their double sum are exact to far
  // below f32's step; rounded down): the scan's squared-L2 scores leave it
  // out, the exact heap scores include it.
  if (qsq) qsq[i] = __double2float_rd(ss * (1.0 - 0x1p-40));
  const double X = (double)__uint_as_float(*xmax_bits);
  const double Q = sqrt(ss);
  const double u = 0x1p-24;
  // fp16 keeps 11 significant bits: each rounded (scaled) operand is within
  // 2^-11 (relative) of its value, so a dot product of rounded operands is
  // within (2^-10 + 2^-22) |q| |x| of the exact one (Cauchy-Schwarz), plus
  // the f32 accumulation of d16 + 2 terms (4 ulps each, allowing
  // truncation). Elements below fp16's normal range (2^-14, scaled) err by at
  // most 2^-25 (scaled) each: 2^-25 sqrt(d) (X / qscale + Q / xscale)
  // unscaled (cosine: unit vectors, scale 1).
  const double c_tc = 0x1p-10 + 0x1p-22 + (double)(d16 + 2) * 0x1p-22;
  const double sub = metric == vrs_exact::kCos ? 0x1p-25 * sqrt((double)d) * 2.0
                                               : 0x1p-25 * sqrt((double)d) * (X / qs + Q / xscale);
  const double g = (double)(d + 4) * u * 1.01;
  double e;
  if (metric == vrs_exact::kCos) {
    e = c_tc + sub + 8.0 * u + 4.0 * g;
  } else if (metric == vrs_exact::kDot) {
    e = (c_tc + 2.0 * g) * Q * X + sub;
  } else {  // squared L2 / Mahalanobis scores |x|^2 - 2 q.x
    e = 2.0 * (c_tc * Q * X + sub) + 8.0 * g * (Q + X) * (Q + X);
    // Folded |x|^2: its hi + lo split (2^-22 relative, or 2^-25 absolute in
    // fp16 units when lo is subnormal) and its share of the accumulation,
    // doubled by the score's factor -2.
    if (fold) e += (0x1p-22 + (double)(d16 + 2) * 0x1p-22) * X * X + 0x1p-24 * ldexp(1.0, fold_m) / xscale;
  }
  absm[i] = (float)(2.0 * e * 1.25) * (1.0f + 0x1p-20f);
}

// Starting bound per query: the k-th smallest pivot-tile minimum plus absm.
// Each tile minimum is the score of a distinct pivot row, so at least k rows
// score <= tau; with k the pivot rank of the proven bound, anything in the
// exact top-k then has approximate score <= tau + absm (a lower rank gives
// the unproven bound that the select checks). With several shards the minima
// are each shard's smallest, all-gathered: the k-th smallest of the union is
// the k-th smallest over every shard's pivot tiles. One block per query.
__global__ void __launch_bounds__(256) tc_tau_kernel(const float* __restrict__ vals, int nparts,
                                                     int64_t part_stride, int len, int nq, int k,
                                                     const float* __restrict__ absm,
                                                     float* __restrict__ init_bound) {
  extern __shared__ Cand buf[];
  __shared__ int s_hist[256];
  __shared__ int s_res[4];
  const int q = blockIdx.x;
  // More minima than shared memory holds: groups of `grp` consecutive
  // minima enter as their minimum (still one distinct row each).
  const int grp = (len + kTauCap / nparts - 1) / (kTauCap / nparts);
  const int glen = (len + grp - 1) / grp;
  const int total = nparts * glen;
  if (total < k) {
    if (threadIdx.x == 0) init_bound[q] = INFINITY;
    return;
  }
  for (int p = 0; p < nparts; p++) {
    const float* row = vals + p * part_stride + (int64_t)q * len;
    for (int t = threadIdx.x; t < glen; t += blockDim.x) {
      float m = INFINITY;
      for (int e = t * grp; e < min(len, t * grp + grp); e++) m = fminf(m, row[e]);
      buf[p * glen + t] = Cand{m, 0u};
    }
  }
  __syncthreads();
  uint32_t kth;
  if (total <= (int)blockDim.x) {
    // Few minima (small shards, e.g. IVF quantisers): one minimum per thread,
    // ranked by counting (ties by position, so the ranks are 0..total-1); the
    // thread of rank k-1 holds the k-th smallest key, the value block_select
    // returns, in one pass instead of four radix passes.
    __shared__ uint32_t s_kth;
    const int t = threadIdx.x;
    if (t < total) {
      const uint32_t mine = ord_key(buf[t].hs);
      int r = 0;
      for (int u = 0; u < total; u++) {
        const uint32_t o = ord_key(buf[u].hs);
        r += (o < mine) || (o == mine && u < t);
      }
      if (r == k - 1) s_kth = mine;
    }
    __syncthreads();
    kth = s_kth;
  } else {
    kth = sel::block_select(buf, total, k, s_hist, s_res);
  }
  if (threadIdx.x == 0) {
    const float tau = ord_inv(kth);
    init_bound[q] = isfinite(tau) ? __fadd_ru(tau, absm[q]) : INFINITY;
  }
}

// The k smallest pivot minima of each query (exactly k values: all below the
// k-th smallest, then copies of it; +inf padding when ntile < k).
__global__ void __launch_bounds__(256) tc_pivot_topk_kernel(const float* __restrict__ tmin, int ntile,
                                                            int nq, int k, float* __restrict__ out) {
  extern __shared__ Cand buf[];
  __shared__ int s_hist[256];
  __shared__ int s_res[4];
  __shared__ int s_pos;
  const int q = blockIdx.x;
  const float* row = tmin + (int64_t)q * ntile;
  float* dst = out + (int64_t)q * k;
  // Groups of consecutive minima beyond the shared capacity (see tc_tau_kernel).
  const int grp = (ntile + kTauCap - 1) / kTauCap;
  const int glen = (ntile + grp - 1) / grp;
  if (glen <= k) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      float m = INFINITY;
      if (j < glen)
        for (int e = j * grp; e < min(ntile, j * grp + grp); e++) m = fminf(m, row[e]);
      dst[j] = m;
    }
    return;
  }
  for (int t = threadIdx.x; t < glen; t += blockDim.x) {
    float m = INFINITY;
    for (int e = t * grp; e < min(ntile, t * grp + grp); e++) m = fminf(m, row[e]);
    buf[t] = Cand{m, 0u};
  }
  if (threadIdx.x == 0) s_pos = 0;
  __syncthreads();
  const uint32_t kth = sel::block_select(buf, glen, k, s_hist, s_res);
  __syncthreads();
  for (int t = threadIdx.x; t < glen; t += blockDim.x) {
    const float v = buf[t].hs;
    if (ord_key(v) < kth) dst[atomicAdd(&s_pos, 1)] = v;
  }
  __syncthreads();
  const float kv = ord_inv(kth);
  for (int j = s_pos + threadIdx.x; j < k; j += blockDim.x) dst[j] = kv;
}

// Gathers every `stride`-th operand row (and |x|^2) into the pivot set.
__global__ void tc_pivot_gather_kernel(const uint16_t* __restrict__ xb, const float* __restrict__ xn,
                                       int64_t m, int64_t stride, int d16,
                                       uint16_t* __restrict__ pb, float* __restrict__ pn) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= m * d16) return;
  int64_t r = i / d16;
  int c = (int)(i - r * d16);
  pb[i] = xb[r * stride * d16 + c];
  if (c == 0 && xn) pn[r] = xn[r * stride];
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 16-bit [rows][d16] row-major, box 64 x box_rows, 128-byte swizzle, zero OOB fill.
int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int d16, bool f16, int box_rows = BM) {
  auto fn = encode_fn();
  if (!fn) {
    set_error(VRS_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
    return VRS_ERR_DRIVER;
  }
  cuuint64_t dims[2] = {(cuuint64_t)d16, (cuuint64_t)std::max<int64_t>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)d16 * 2};
  cuuint32_t box[2] = {(cuuint32_t)KBW, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(VRS_ERR_DRIVER, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return VRS_ERR_DRIVER;
  }
  return VRS_OK;
}

}  // namespace

bool tc_supported(int metric, int d) {
  return d >= 1 && d <= 128 &&
         (metric == vrs_exact::kL2 || metric == vrs_exact::kMaha || metric == vrs_exact::kDot ||
          metric == vrs_exact::kCos);
}

int tc_d16(int metric, int d) { return (tc_fold(metric, d) ? d + 2 + 15 : d + 15) / 16 * 16; }

int tc_base_prep(const float* x, int64_t n, int d, int dp, int metric, float xscale, int fold_m, void* xb,
                 float* xn, unsigned int* xmax_bits, uint32_t* tiny, int* n_tiny, int tiny_cap, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  tc_base_prep_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(
      x, n, d, dp, tc_d16(metric, d), metric, xscale, fold_m, (uint16_t*)xb, xn, xmax_bits, tiny, n_tiny,
      tiny_cap);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int tc_query_prep(const float* q_in, int nq, int d, int dp, int metric, const unsigned int* xmax_bits,
                  float xscale, int fold_m, float* qpad, float* qaux, void* qb, float* qscale, float* absm,
                  int* overflow, float* qsq, cudaStream_t s) {
  if (nq == 0) return VRS_OK;
  if (d > 128) {
    set_error(VRS_ERR_INVALID_CONFIG, "tensor-core query prep needs d <= 128");
    return VRS_ERR_INVALID_CONFIG;
  }
  tc_query_prep_kernel<<<(nq + kPrepWarps - 1) / kPrepWarps, kPrepWarps * 32, 0, s>>>(
      q_in, nq, d, dp, tc_d16(metric, d), metric, xmax_bits, xscale, fold_m, qpad, qaux, (uint16_t*)qb, qscale,
      absm, overflow, qsq);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int tc_pivot_gather(const void* xb, const float* xn, int64_t m, int64_t stride, int d16, void* pb,
                    float* pn, cudaStream_t s) {
  if (m == 0) return VRS_OK;
  const int64_t total = m * d16;
  tc_pivot_gather_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      (const uint16_t*)xb, xn, m, stride, d16, (uint16_t*)pb, pn);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int tc_tau(const float* vals, int nparts, int64_t part_stride, int len, int nq, int k, const float* absm,
           float* init_bound, cudaStream_t s) {
  if (nq == 0) return VRS_OK;
  if (nparts > kTauCap) {
    set_error(VRS_ERR_INVALID_CONFIG, "too many shards for the pooled pivot");
    return VRS_ERR_INVALID_CONFIG;
  }
  const int grp = (len + kTauCap / nparts - 1) / (kTauCap / nparts);
  const size_t smem = (size_t)std::max(nparts * ((len + grp - 1) / grp), 1) * sizeof(Cand);
  VRS_CUDA(cudaFuncSetAttribute(tc_tau_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  tc_tau_kernel<<<nq, 256, smem, s>>>(vals, nparts, part_stride, len, nq, k, absm, init_bound);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int tc_pivot_topk(const float* tmin, int ntile, int nq, int k, float* out, cudaStream_t s) {
  if (nq == 0) return VRS_OK;
  const int grp = (ntile + kTauCap - 1) / kTauCap;
  const size_t smem = (size_t)std::max((ntile + grp - 1) / grp, 1) * sizeof(Cand);
  VRS_CUDA(cudaFuncSetAttribute(tc_pivot_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  tc_pivot_topk_kernel<<<nq, 256, smem, s>>>(tmin, ntile, nq, k, out);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

TcPlan tc_plan(int64_t n, int nq, int kk, int num_sms, int align_tiles) {
  TcPlan p;
  p.qtiles = (nq + BM * NACC - 1) / (BM * NACC);
  p.cap = 1024;
  while (p.cap < 2 * kk + 2 * BN) p.cap *= 2;
  const int64_t ntile_total = (n + BN - 1) / BN;
  double best = 1e30;
  p.nseg = 1;
  for (int s = 1; s <= 16; s++) {
    if (s > 1 && ntile_total / s < 8) break;
    const double waves = (double)p.qtiles * s / num_sms;
    const double cost = std::ceil(waves) / waves + 0.003 * s;
    if (cost < best - 1e-9) {
      best = cost;
      p.nseg = s;
    }
  }
  int64_t tiles_per_seg = (ntile_total + p.nseg - 1) / p.nseg;
  tiles_per_seg = (tiles_per_seg + align_tiles - 1) / align_tiles * align_tiles;
  p.seg_len = std::max<int64_t>(1, tiles_per_seg) * BN;
  p.nseg = (int)std::max<int64_t>(1, (n + p.seg_len - 1) / p.seg_len);
  return p;
}

// Plan of the 2-SM candidate pass: pairs of 256 queries x segments of
// 256-row tiles, at most 8 segments (4 lists each: the warp select takes at
// most 32 lists per query), chosen like tc_plan for whole waves of SM pairs.
TcPlan tc_plan2(int64_t n, int nq, int kk, int num_sms, int align_tiles) {
  TcPlan p;
  p.qtiles = (nq + 2 * P_BM - 1) / (2 * P_BM);
  p.cap = 1024;
  while (p.cap < 2 * kk + 2 * BN) p.cap *= 2;
  const int pairs = std::max(1, num_sms / 2);
  const int64_t ntile_total = (n + P_BN - 1) / P_BN;
  double best = 1e30;
  p.nseg = 1;
  for (int s = 1; s <= 8; s++) {
    if (s > 1 && ntile_total / s < 4) break;
    const double waves = (double)p.qtiles * s / pairs;
    const double cost = std::ceil(waves) / waves + 0.003 * s;
    if (cost < best - 1e-9) {
      best = cost;
      p.nseg = s;
    }
  }
  int64_t tiles_per_seg = std::max<int64_t>(1, (ntile_total + p.nseg - 1) / p.nseg);
  tiles_per_seg = (tiles_per_seg + align_tiles - 1) / align_tiles * align_tiles;
  p.seg_len = tiles_per_seg * P_BN;
  p.nseg = (int)std::max<int64_t>(1, (n + p.seg_len - 1) / p.seg_len);
  return p;
}

// Candidate pass on CTA pairs (knn_scan_tc2_kernel): lists [4 * nseg][nq][cap].
int tc_scan2(const void* qb, int nq_rows_alloc, const void* xb, int64_t n, int d, const float* xn, int metric,
             int nq, int kk, const TcPlan& p, Cand* cand, int* cnt, int* overflow, const float* absm, int* err,
             float* tmin, const float* init_bound, const float* qscale, float xscale, cudaStream_t s) {
  if (n == 0 || nq == 0) return VRS_OK;
  if (nq_rows_alloc % (2 * P_BM) != 0) {
    set_error(VRS_ERR_INVALID_CONFIG, "2-SM scan: query operand rows must be a multiple of 256");
    return VRS_ERR_INVALID_CONFIG;
  }
  const int d16 = tc_d16(metric, d);
  CUtensorMap tmA, tmB;
  const bool f16 = tc_fp16(metric);
  VRS_TRY(make_tmap(&tmA, qb, nq_rows_alloc, d16, f16));
  VRS_TRY(make_tmap(&tmB, xb, n, d16, f16, P_HALF));
  TcScanArgs a;
  a.xn = xn;
  a.n = n;
  a.nq = nq;
  a.ksteps = d16 / 16;
  a.kblk = (d16 + KBW - 1) / KBW;
  a.seg_len = p.seg_len;
  a.cand = cand;
  a.cnt = cnt;
  a.overflow = overflow;
  a.cap = p.cap;
  a.k = kk;
  a.absm = absm;
  a.err = err;
  a.tmin = tmin;
  a.tmin_stride = tc_pivot_values2(n);
  if (tmin && p.seg_len % ((int64_t)kPivotGroup * P_BN) != 0) {
    set_error(VRS_ERR_INVALID_CONFIG, "pivot segments must start on pivot-group boundaries");
    return VRS_ERR_INVALID_CONFIG;
  }
  a.idesc = f16 ? idesc_f16(2 * P_BM, P_BN) : idesc_bf16(2 * P_BM, P_BN);
  a.qscale = qscale;
  a.xscale = xscale;
  a.init_bound = init_bound;
  const bool l2 = metric == vrs_exact::kL2 || metric == vrs_exact::kMaha;
  auto kern = tc_fold(metric, d) ? (tmin ? knn_scan_tc2_kernel<2, true> : knn_scan_tc2_kernel<2, false>)
              : l2               ? (tmin ? knn_scan_tc2_kernel<0, true> : knn_scan_tc2_kernel<0, false>)
                                 : (tmin ? knn_scan_tc2_kernel<1, true> : knn_scan_tc2_kernel<1, false>);
  static std::once_flag attr_once[64];
  int dev = 0;
  VRS_CUDA(cudaGetDevice(&dev));
  int attr_err = 0;
  if (dev < 64) {
    std::call_once(attr_once[dev], [&] {
      for (auto f : {knn_scan_tc2_kernel<0, false>, knn_scan_tc2_kernel<1, false>, knn_scan_tc2_kernel<2, false>,
                     knn_scan_tc2_kernel<0, true>, knn_scan_tc2_kernel<1, true>, knn_scan_tc2_kernel<2, true>})
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM_TOTAL) != cudaSuccess)
          attr_err = 1;
    });
  } else {
    VRS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM_TOTAL));
  }
  if (attr_err) {
    set_error(VRS_ERR_DRIVER, "cudaFuncSetAttribute(knn_scan_tc2_kernel) failed");
    return VRS_ERR_DRIVER;
  }
  dim3 grid(2 * p.qtiles, p.nseg);  // x: two CTAs (one cluster) per 256 queries
  kern<<<grid, THREADS, P_SMEM_TOTAL, s>>>(tmA, tmB, a);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int tc_scan(const void* qb, int nq_rows_alloc, const void* xb, int64_t n, int d, const float* xn,
            int metric, int nq, int kk, const TcPlan& p, Cand* cand, int* cnt, int* overflow,
            const float* absm, int* err, float* tmin, const float* init_bound, const float* qscale, float xscale,
            cudaStream_t s) {
  if (n == 0 || nq == 0) return VRS_OK;
  const int d16 = tc_d16(metric, d);
  CUtensorMap tmA, tmB;
  const bool f16 = tc_fp16(metric);
  VRS_TRY(make_tmap(&tmA, qb, nq_rows_alloc, d16, f16));
  VRS_TRY(make_tmap(&tmB, xb, n, d16, f16));
  TcScanArgs a;
  a.xn = xn;
  a.n = n;
  a.nq = nq;
  a.ksteps = d16 / 16;
  a.kblk = (d16 + KBW - 1) / KBW;
  a.seg_len = p.seg_len;
  a.cand = cand;
  a.cnt = cnt;
  a.overflow = overflow;
  a.cap = p.cap;
  a.k = kk;
  a.absm = absm;
  a.err = err;
  a.tmin = tmin;
  a.tmin_stride = 2 * tc_pivot_groups(n);
  if (tmin && p.seg_len % ((int64_t)kPivotGroup * BN) != 0) {
    set_error(VRS_ERR_INVALID_CONFIG, "pivot segments must start on pivot-group boundaries");
    return VRS_ERR_INVALID_CONFIG;
  }
  a.idesc = f16 ? idesc_f16(BM, BN) : idesc_bf16(BM, BN);
  a.qscale = qscale;
  a.xscale = xscale;
  a.init_bound = init_bound;
  const bool l2 = metric == vrs_exact::kL2 || metric == vrs_exact::kMaha;
  auto kern = tc_fold(metric, d) ? (tmin ? knn_scan_tc_kernel<2, true> : knn_scan_tc_kernel<2, false>)
              : l2               ? (tmin ? knn_scan_tc_kernel<0, true> : knn_scan_tc_kernel<0, false>)
                                 : (tmin ? knn_scan_tc_kernel<1, true> : knn_scan_tc_kernel<1, false>);
  static std::once_flag attr_once[64];
  int dev = 0;
  VRS_CUDA(cudaGetDevice(&dev));
  int attr_err = 0;
  if (dev < 64) {
    std::call_once(attr_once[dev], [&] {
      for (auto f : {knn_scan_tc_kernel<0, true>, knn_scan_tc_kernel<0, false>, knn_scan_tc_kernel<1, true>,
                     knn_scan_tc_kernel<1, false>, knn_scan_tc_kernel<2, true>, knn_scan_tc_kernel<2, false>})
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL) !=
            cudaSuccess)
          attr_err = 1;
    });
  } else {
    VRS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL));
  }
  if (attr_err) {
    set_error(VRS_ERR_DRIVER, "cudaFuncSetAttribute(knn_scan_tc_kernel) failed");
    return VRS_ERR_DRIVER;
  }
  dim3 grid(p.qtiles, p.nseg);
  kern<<<grid, THREADS, SMEM_TOTAL, s>>>(tmA, tmB, a);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

}  // namespace tc
}  // namespace vrs
