// kmeans_tc.cu -- tensor-core (tcgen05) k-means assignment for the GEMM-form
// metrics (squared L2, Mahalanobis, dot, cosine).
//
// Persistent CTAs loop over tiles of 256 points (two M=128 fp16 operand
// tiles, loaded by TMA, double-buffered); the K centroids stream as 128-row
// fp16 tiles through a TMA ring of 64-column k-block slots; one thread
// issues tcgen05.mma (kind::f16) into two 128x128 f32 TMEM accumulators
// (double-buffered). Sixteen epilogue warps
// (one thread = one point, two warps per point splitting each tile's
// columns) keep the approximate best score and every group of four
// centroids whose smallest approximate score is within the point's bound
// (up to kGroupSlots groups per column half, stored straight to global
// memory, plus the smallest group minimum that did not fit, so a point
// whose dropped group may hold its nearest centroid is flagged for an exact
// scan). kmeans_finalize then picks the exact argmin among those
// candidates in the reference's f32 arithmetic (find_nearest,
// crates/vector-cuda/src/kmeans.rs:361-407: strict comparison, lowest index
// wins ties) and records the exact distance for the inertia.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "tc_common.cuh"
#include "vrs_exact.cuh"
#include "vrs_exact_lanes.cuh"
#include "vrs_internal.cuh"
#include "vrs_kmeans_tc.cuh"
#include "vrs_select.cuh"

namespace vrs {
namespace kmtc {
namespace {

using namespace vrs::tc;

// ABUF point-tile buffers: the next point tile's operands load while the
// current one's MMAs run (one buffer left the tensor pipe idle through every
// reload, K / BN tiles apart). The centroid tiles come from L2 through a
// ring of SLOTS slots of one 64-column k-block each: a slot frees as soon as
// the MMAs of its k-block complete, so each load is issued up to SLOTS - 1
// k-blocks of MMA time before it is needed.
#ifndef KM_SLOTS
#define KM_SLOTS 6
#endif
constexpr int BM = 128, NACC = 2, BN = 128, KBW = 64, MAX_KBLK = 2, SLOTS = KM_SLOTS, ABUF = 2;
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr int HALF_COLS = BN / 2;
constexpr int NG = kGroupSlots;
constexpr uint32_t BLK = BM * 128;
constexpr size_t SMEM_A = (size_t)ABUF * NACC * MAX_KBLK * BLK;
constexpr size_t SMEM_B = (size_t)SLOTS * BLK;
constexpr size_t SMEM_CN = 2 * BN * sizeof(float);  // |c|^2 of the tile in each TMEM buffer
constexpr size_t SMEM_BAR = 256;
constexpr size_t SMEM_TOTAL = 1024 + SMEM_A + SMEM_B + SMEM_CN + SMEM_BAR;
static_assert(SMEM_TOTAL <= 232448, "dynamic shared memory above the 227 KB per-block limit");
static_assert((2 * SLOTS + 5 + 2 * ABUF) * 8 + 8 <= SMEM_BAR, "barrier region too small");
static_assert(SLOTS >= 2, "the ring needs two slots");
constexpr uint64_t WAIT_NS = 2000000000ull;
constexpr uint32_t TMEM_COLS = 512;

struct AssignArgs {
  const float* cn;          // |c|^2 per centroid (L2 mode), zero padded
  const float* xq;          // |x| per point (margins)
  const unsigned int* cmax; // max |c| (float bits)
  int64_t n;
  int k;
  int d;
  int ksteps, kblk;
  int mode;                 // 0: score |c|^2 - 2 x.c ; 1: score -x.c
  int metric;
  float acc_scale;          // 1 / (operand scale)^2: unscales the accumulator
  float inv_scale;          // 1 / operand scale (margins)
  Res* res;                 // [n][2] per (point, column half)
  Groups groups;            // candidate groups, [n][2][NG] slots
  int* err;
  // Upper bound on each point's best approximate score (MODE 0, from the
  // previous Lloyd step; null: none): candidates start within it.
  const float* init_bound;
};

// Acceptance margin of one point in score units (same bound as the kNN
// path, with the centroids as the "base"). Operands are fp16 of the values
// times a power-of-two scale s (largest element in [2^13, 2^14)): fp16 keeps
// 11 significant bits, so each product of rounded operands is within
// 2^-10 + 2^-22 (relative) of the exact one; elements below fp16's normal
// range add at most 2^-25 each in scaled units, i.e. 2^-25 sqrt(d) |other| / s
// per side after unscaling; plus the f32 accumulation of d16 + 2 terms
// (4 ulps each, allowing truncation). rd = sqrt((double)d), computed once
// by the caller (correctly rounded, so every kernel gets the same margin).
__device__ __forceinline__ float point_margin(int metric, int d, double rd, float Q, float X, float inv_s) {
  const double u = 0x1p-24;
  const int d16 = (d + 15) / 16 * 16;
  const double c_tc = 0x1p-10 + 0x1p-22 + (double)(d16 + 2) * 0x1p-22;
  const double sub = 0x1p-25 * rd * ((double)Q + X) * (double)inv_s;
  const double g = (double)(d + 4) * u * 1.01;
  double e;
  if (metric == vrs_exact::kCos) {  // unit vectors, s = 1
    e = c_tc + 0x1p-25 * rd * 2.0 + 8.0 * u + 4.0 * g;
  } else if (metric == vrs_exact::kDot) {
    e = (c_tc + 2.0 * g) * (double)Q * (double)X + sub;
  } else {
    e = 2.0 * (c_tc * (double)Q * (double)X + sub) + 8.0 * g * ((double)Q + X) * ((double)Q + X);
  }
  return (float)(2.0 * e * 1.25) * (1.0f + 0x1p-20f);
}

// MODE 0: score = |c|^2 - 2 x.c (squared L2, Mahalanobis); MODE 1: score =
// -x.c (dot, cosine on unit rows).
template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    kmeans_assign_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            AssignArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + SMEM_A;
  float* s_cn = (float*)(sB + SMEM_B);  // [2][BN]
  uint64_t* bars = (uint64_t*)((uint8_t*)s_cn + SMEM_CN);
  uint64_t* full = bars;
  uint64_t* empty = bars + SLOTS;
  uint64_t* tfull = bars + 2 * SLOTS;
  uint64_t* tempty = tfull + 2;
  uint64_t* afull = tempty + 2;   // [ABUF]
  uint64_t* aempty = afull + ABUF;  // [ABUF]
  uint64_t* drain = aempty + ABUF;  // abort path: all issued MMAs complete
  uint32_t* s_tmem = (uint32_t*)(drain + 1);
  volatile int* s_abort = (volatile int*)(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nptiles = (int)((a.n + BM * NACC - 1) / (BM * NACC));
  const int kt = (a.k + BN - 1) / BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SLOTS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    for (int b = 0; b < ABUF; b++) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(drain, 1);
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
    if (lane == 0) {
      // Point tile of local index lp goes to A buffer lp % ABUF; its use
      // number u = lp / ABUF waits for the buffer's previous phase.
      auto load_a = [&](int pt, int lp) -> bool {
        const int ab = lp % ABUF, u = lp / ABUF;
        if (!mbar_wait(&aempty[ab], (u & 1) ^ 1, s_abort, a.err, 11, WAIT_NS)) return false;
        mbar_expect_tx(&afull[ab], (uint32_t)(NACC * a.kblk) * BLK);
        for (int acc = 0; acc < NACC; acc++)
          for (int kb = 0; kb < a.kblk; kb++)
            tma_load_2d(sA + ((ab * NACC + acc) * MAX_KBLK + kb) * BLK, &tmA, kb * KBW,
                        pt * BM * NACC + acc * BM, &afull[ab]);
        return true;
      };
      uint32_t q = 0;  // k-blocks queued so far: slot q % SLOTS, use q / SLOTS
      int lp = 0;
      bool ok = blockIdx.x >= nptiles || load_a(blockIdx.x, 0);
      for (int pt = blockIdx.x; ok && pt < nptiles; pt += gridDim.x, lp++) {
        // The next point tile's operands go into the buffer of the tile
        // before this one, free once that tile's MMAs complete: issued as
        // soon as a non-blocking test sees it free, so the centroid tiles
        // keep flowing meanwhile (waiting for it held the ring one tile
        // deep at every point-tile boundary); at the tile's last centroid
        // tile at the latest.
        bool a_next = pt + (int)gridDim.x >= nptiles;
        const int nb = (lp + 1) % ABUF;
        const uint32_t npar = (uint32_t)(((lp + 1) / ABUF) & 1) ^ 1u;
        for (int j = 0; ok && j < kt; j++) {
          for (int kb = 0; kb < a.kblk; kb++, q++) {
            const int s = (int)(q % SLOTS);
            if (!mbar_wait(&empty[s], ((q / SLOTS) & 1) ^ 1, s_abort, a.err, 12, WAIT_NS)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&full[s], BLK);
            tma_load_2d(sB + s * BLK, &tmB, kb * KBW, j * BN, &full[s]);
          }
          if (ok && !a_next && (j == kt - 1 || mbar_test(&aempty[nb], npar))) {
            if (!load_a(pt + gridDim.x, lp + 1)) ok = false;
            a_next = true;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BM, BN);
      // Descriptors differ only in the masked start-address field: the A
      // ones are formed per point tile (for its buffer), the B ones per
      // slot.
      const DescSw128 a_desc(sA), b_desc(sB);
      const int ksteps = a.ksteps, kblk = a.kblk;
      uint32_t g = 0;  // centroid tiles issued: TMEM buffer g & 1
      uint32_t q = 0;  // k-blocks consumed: slot q % SLOTS
      int lp = 0;
      bool ok = true, issued = false;
      for (int pt = blockIdx.x; ok && pt < nptiles; pt += gridDim.x, lp++) {
        const int ab = lp % ABUF, u = lp / ABUF;
        uint64_t ad[NACC][MAX_KBLK * 4];
#pragma unroll
        for (int acc = 0; acc < NACC; acc++)
#pragma unroll
          for (int ks = 0; ks < MAX_KBLK * 4; ks++)
            ad[acc][ks] = a_desc.at((uint32_t)((ab * NACC + acc) * MAX_KBLK * BLK + (ks >> 2) * BLK +
                                               (ks & 3) * 32) >> 4);
        if (!mbar_wait(&afull[ab], u & 1, s_abort, a.err, 13, WAIT_NS)) break;
        tc_fence_after();
        for (int j = 0; j < kt; j++, g++) {
          const int b = g & 1;
          if (!mbar_wait(&tempty[b], ((g >> 1) & 1) ^ 1, s_abort, a.err, 15, WAIT_NS)) {
            ok = false;
            break;
          }
          if (MODE == 0) {
            // |c|^2 of this tile's centroids rides on the same barrier as
            // the accumulator (cn is zero padded to whole tiles + 128).
            mbar_expect_tx_only(&tfull[b], BN * sizeof(float));
            bulk_copy_g2s(s_cn + b * BN, a.cn + (int64_t)j * BN, BN * sizeof(float), &tfull[b]);
          }
#pragma unroll
          for (int kb = 0; kb < MAX_KBLK; kb++) {
            if (kb >= kblk) break;
            const int s = (int)(q % SLOTS);
            if (!mbar_wait(&full[s], (q / SLOTS) & 1, s_abort, a.err, 14, WAIT_NS)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int acc = 0; acc < NACC; acc++) {
              const uint32_t d = tmem + acc * 256 + b * BN;
#pragma unroll
              for (int ks = 0; ks < 4; ks++)
                if (kb * 4 + ks < ksteps)
                  mma_f16(d, ad[acc][kb * 4 + ks], b_desc.at((uint32_t)(s * BLK + ks * 32) >> 4), idesc,
                          kb * 4 + ks > 0 ? 1u : 0u);
            }
            issued = true;
            mma_commit(&empty[s]);
            q++;
          }
          if (!ok) break;
          mma_commit(&tfull[b]);
        }
        if (ok) mma_commit(&aempty[ab]);
      }
      if (*s_abort && issued) {
        // A tile may have stopped between k-blocks: wait (bounded) for every
        // MMA issued so far before the TMEM is released.
        volatile int dummy = 0;
        mma_commit(drain);
        mbar_wait(drain, 0, &dummy, a.err, 0, WAIT_NS / 4);
      }
    }
  } else {
    // ---------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int acc = (ew >> 2) & 1;
    const int ch = ew >> 3;
    const int quad = warp & 3;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const float X = __uint_as_float(*a.cmax);
    const double rd = sqrt((double)a.d);
    // The point's |x| and starting bound for the next point tile are loaded
    // one tile ahead, off the path between the MMAs and this warp.
    const int64_t poff = acc * BM + quad * 32 + lane;
    auto load_point = [&](int pt, float* xq, float* ib) {
      const int64_t p = (int64_t)pt * BM * NACC + poff;
      const bool in = pt < nptiles && p < a.n;
      *xq = in ? a.xq[p] : 0.0f;
      *ib = in && a.init_bound ? a.init_bound[p] : INFINITY;
    };
    float nxq, nib;
    load_point(blockIdx.x, &nxq, &nib);
    uint32_t g = 0;
    bool ok = true;
    for (int pt = blockIdx.x; ok && pt < nptiles; pt += gridDim.x) {
      const int64_t p = (int64_t)pt * BM * NACC + poff;
      const bool vp = p < a.n;
      const float pxq = nxq, pib = nib;
      load_point(pt + gridDim.x, &nxq, &nib);
      const float absm = vp ? point_margin(a.metric, a.d, rd, pxq, X, a.inv_scale) : 0.0f;
      const float f2 = -2.0f * a.acc_scale, f1 = -a.acc_scale;
      float best = INFINITY;
      // Padding points keep nothing; with a starting bound s (>= the exact
      // score of some centroid), best approx <= s + e and e < absm / 2, so
      // s + 1.5 absm >= best approx + absm keeps every candidate the
      // unbounded sweep would keep at the end.
      float bound = !vp ? -INFINITY : a.init_bound ? __fadd_ru(pib, 1.5f * absm) : INFINITY;
      float lost = INFINITY;  // smallest minimum of a group that found the slots full
      int cnt = 0;            // groups kept
      const int64_t slot0 = (p * 2 + ch) * NG;
      for (int j = 0; j < kt; j++, g++) {
        const int b = g & 1;
        const bool w = mbar_wait(&tfull[b], (g >> 1) & 1, s_abort, a.err, 16, WAIT_NS);
        if (!__all_sync(sel::kFull, w)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int c0 = j * BN + ch * HALF_COLS;
        const int rem = a.k - c0;
        const int valid = rem < HALF_COLS ? (rem > 0 ? rem : 0) : HALF_COLS;
#pragma unroll 1
        for (int c = 0; c < HALF_COLS / 32; c++) {
          float v[32];
          tmem_ld32(tmem + lane_base + acc * 256 + b * BN + ch * HALF_COLS + c * 32, v);
          const int cb = valid - c * 32;
          // scores, smaller is better
          if (MODE == 0) {
            const float4* cp = reinterpret_cast<const float4*>(s_cn + b * BN + ch * HALF_COLS + c * 32);
#pragma unroll
            for (int j4 = 0; j4 < 8; j4++) {
              const float4 x4 = cp[j4];
              v[4 * j4 + 0] = fmaf(f2, v[4 * j4 + 0], x4.x);
              v[4 * j4 + 1] = fmaf(f2, v[4 * j4 + 1], x4.y);
              v[4 * j4 + 2] = fmaf(f2, v[4 * j4 + 2], x4.z);
              v[4 * j4 + 3] = fmaf(f2, v[4 * j4 + 3], x4.w);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = f1 * v[i];
          }
          if (c == HALF_COLS / 32 - 1) {
            // The tile's last columns are in registers and its |c|^2 read:
            // hand the TMEM buffer (and its |c|^2 slot) back to the MMA
            // issuer before the selection work.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
          if (cb < 32) {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (i >= cb) v[i] = INFINITY;
          }
          float gm[8];
#pragma unroll
          for (int i = 0; i < 8; i++) gm[i] = fmin3(v[4 * i], v[4 * i + 1], fminf(v[4 * i + 2], v[4 * i + 3]));
          const float cmn = fmin3(fmin3(gm[0], gm[1], gm[2]), fmin3(gm[3], gm[4], gm[5]), fminf(gm[6], gm[7]));
          // Padding points have bound -inf and never hit; a chunk of
          // columns past K only (+inf) never hits either. Most chunks hold
          // no candidate of any of the warp's points: one vote skips them.
          const bool hit = cmn <= bound && cmn < INFINITY;
          if (__any_sync(sel::kFull, hit) && hit) {
            // A better chunk minimum tightens the bound. Groups already
            // kept stay; the triage filters their scores by the final
            // bound.
            if (cmn < best) {
              best = cmn;
              bound = fminf(bound, __fadd_ru(best, absm));
            }
            // Each group of four whose minimum passes: its four scores in
            // one 16-byte store and its first column (static register
            // indices, predicated; only a warp's hitting lanes run this).
            // Columns past K inside a kept group score +inf and are never
            // chosen.
#pragma unroll
            for (int i = 0; i < 8; i++) {
              if (gm[i] <= bound) {
                if (cnt < NG) {
                  a.groups.sc[slot0 + cnt] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                  a.groups.col[slot0 + cnt] = (uint32_t)(c0 + c * 32 + 4 * i);
                  cnt++;
                } else {
                  lost = fminf(lost, gm[i]);
                }
              }
            }
            if (cnt >= NG - 1) {
              // Make room for the next hit (rarely needed): drop kept groups
              // the bound has passed. This thread wrote the slots, so it
              // reads them back; the chunk's scores are no longer live.
              int k2 = 0;
              for (int e = 0; e < cnt; e++) {
                const float4 s4 = a.groups.sc[slot0 + e];
                if (fminf(fminf(s4.x, s4.y), fminf(s4.z, s4.w)) <= bound) {
                  if (k2 != e) {
                    a.groups.sc[slot0 + k2] = s4;
                    a.groups.col[slot0 + k2] = a.groups.col[slot0 + e];
                  }
                  k2++;
                }
              }
              cnt = k2;
            }
          }
        }
      }
      if (!ok) break;
      if (vp) {
        Res r;
        r.best = best;
        r.bi = 0;
        r.cnt = cnt;
        r.lost = lost;
        a.res[p * 2 + ch] = r;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Finalize, step 1 (one thread per point): the bound from the point's two
// records. The exact nearest centroid c* is always within it: its
// approximate score is at most exact(c*) + e <= exact(best approximate) + e
// <= best approximate + 2e < bound, and it was kept unless a full buffer
// pushed out something within the bound. So
//  * a candidate pushed out within the bound (or a near-zero cosine point)
//    -> list F (flags[0] = count, indices from flags + 2): all K centroids
//    scored exactly;
//  * exactly one candidate within the bound -> it is c*: assigned here, no
//    exact distance (kmeans_dist_kernel fills distances in after the loop);
//  * several -> list M (flags[1] = count, indices from flags + 2 + n):
//    scored exactly by kmeans_multi_kernel.
// Appends `value` to two lists (list0 for the threads with `take` == 1,
// list1 for `take` == 2) with one global atomic per block and list: warps
// count by ballot, a shared prefix orders the warps, thread 0 reserves the
// block's range. Every thread of the block must call (blockDim = 256).
__device__ __forceinline__ void block_append2(int* counter0, int* list0, int* counter1, int* list1, int take,
                                              int value) {
  __shared__ int s_cnt[2][8];
  __shared__ int s_base[2];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  const unsigned m0 = __ballot_sync(0xffffffffu, take == 1), m1 = __ballot_sync(0xffffffffu, take == 2);
  if (lane == 0) {
    s_cnt[0][w] = __popc(m0);
    s_cnt[1][w] = __popc(m1);
  }
  __syncthreads();
  if (threadIdx.x < 2) {
    int tot = 0;
    for (int i = 0; i < 8; i++) {
      const int c = s_cnt[threadIdx.x][i];
      s_cnt[threadIdx.x][i] = tot;  // exclusive prefix over the warps
      tot += c;
    }
    s_base[threadIdx.x] = tot ? atomicAdd(threadIdx.x ? counter1 : counter0, tot) : 0;
  }
  __syncthreads();
  if (take == 1) list0[s_base[0] + s_cnt[0][w] + __popc(m0 & below)] = value;
  if (take == 2) list1[s_base[1] + s_cnt[1][w] + __popc(m1 & below)] = value;
}

template <int METRIC>
__global__ void __launch_bounds__(256) kmeans_triage_kernel(
    int64_t n, int d, const float* __restrict__ xq, const unsigned int* __restrict__ cmax,
    const Res* __restrict__ res, Groups groups, const int* __restrict__ force_full,
    int32_t* __restrict__ assign, int* __restrict__ flags, float inv_scale, float* __restrict__ pscore) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int cls = 0;  // 0: assigned here (or past the end), 1: list F, 2: list M
  if (i < n) {
    const Res r0 = res[i * 2], r1 = res[i * 2 + 1];
    const float absm = point_margin(METRIC, d, sqrt((double)d), xq[i], __uint_as_float(*cmax), inv_scale);
    const float bound = __fadd_ru(fminf(r0.best, r1.best), absm);
    if (r0.lost <= bound || r1.lost <= bound || (force_full && force_full[i])) {
      cls = 1;
      if (pscore) pscore[i] = INFINITY;  // full exact scan: no approximate score kept
    } else {
      int nin = 0;
      uint32_t only = 0;
      float only_hs = 0.0f;
      for (int h = 0; h < 2; h++) {
        const Res r = h ? r1 : r0;
        for (int e = 0; e < r.cnt; e++) {
          const int64_t sl = (i * 2 + h) * NG + e;
          const float4 s4 = groups.sc[sl];
          const uint32_t col = groups.col[sl];
          const float sc[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int jj = 0; jj < 4; jj++) {
            if (sc[jj] <= bound) {
              nin++;
              only = col + jj;
              only_hs = sc[jj];
            }
          }
        }
      }
      if (nin == 1) {
        assign[i] = (int)only;
        // exact score of the assigned centroid <= approx + e, e < absm / 2
        if (pscore) pscore[i] = __fadd_ru(only_hs, 0.5f * absm);
      } else {
        cls = 2;
      }
    }
  }
  // The lists' order is immaterial: every listed point is scored on its own.
  block_append2(&flags[0], flags + 2, &flags[1], flags + 2 + n, cls, (int)i);
}

// Finalize, step 2: the points of list M, one half-warp per point (its 16
// lanes are the reference's 16 SIMD lanes), striding over the list. Lane l
// loads group slot l & 7 of column half l >> 3, so all of a point's groups
// are read at once; the scores within the bound are then taken two at a
// time (lowest lane, lowest column first) and scored exactly (rank_key2:
// both rows' loads in flight) for the exact argmin, lowest index on ties,
// with the exact distance.
template <int METRIC>
__global__ void __launch_bounds__(128) kmeans_multi_kernel(
    const float* __restrict__ x, int64_t n, int d, int dp, const float* __restrict__ cent,
    const float* __restrict__ cent_aux, const float* __restrict__ x_aux, const float* __restrict__ xq,
    const unsigned int* __restrict__ cmax, const Res* __restrict__ res, Groups groups,
    const int* __restrict__ flags, int32_t* __restrict__ assign, float* __restrict__ dist, float inv_scale,
    float* __restrict__ pscore) {
  static_assert(2 * NG == 16, "one group slot per lane of a half-warp");
  const int hl = threadIdx.x & 15;
  const int hsh = threadIdx.x & 16;
  const unsigned mask = 0xffffu << hsh;
  const bool hib = vrs_exact::higher_is_better(METRIC);
  const int count = flags[1];
  const int* list = flags + 2 + n;
  const int64_t nhw = ((int64_t)gridDim.x * blockDim.x) >> 4;
  for (int64_t f = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4; f < count; f += nhw) {
    const int64_t i = list[f];
    const float* v = x + i * dp;
    const float va = METRIC == vrs_exact::kCos ? x_aux[i] : 0.0f;
    const Res r0 = res[i * 2], r1 = res[i * 2 + 1];
    const float absm = point_margin(METRIC, d, sqrt((double)d), xq[i], __uint_as_float(*cmax), inv_scale);
    const float bound = __fadd_ru(fminf(r0.best, r1.best), absm);
    const int h = hl >> 3, e = hl & 7;
    float4 s4 = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
    uint32_t col = 0;
    if (e < (h ? r1.cnt : r0.cnt)) {
      s4 = groups.sc[(i * 2 + h) * NG + e];
      col = groups.col[(i * 2 + h) * NG + e];
    }
    // This lane's scores within the bound, one bit per column of its group.
    unsigned mine = (s4.x <= bound ? 1u : 0u) | (s4.y <= bound ? 2u : 0u) | (s4.z <= bound ? 4u : 0u) |
                    (s4.w <= bound ? 8u : 0u);
    // Next candidate (id, approximate score): the lowest remaining bit of
    // the lowest lane that has one; false when none is left.
    auto next = [&](uint32_t* id, float* hs) -> bool {
      const unsigned lm = (__ballot_sync(mask, mine != 0) >> hsh) & 0xffffu;
      if (!lm) return false;
      const int l = __ffs(lm) - 1;
      const int jb = __ffs(__shfl_sync(mask, mine, l, 16)) - 1;
      const float sv = jb == 0 ? s4.x : jb == 1 ? s4.y : jb == 2 ? s4.z : s4.w;
      *hs = __shfl_sync(mask, sv, l, 16);
      *id = __shfl_sync(mask, col, l, 16) + (uint32_t)jb;
      if (hl == l) mine &= mine - 1;
      return true;
    };
    int best = 0x7fffffff;
    float best_key = hib ? -INFINITY : INFINITY;
    float best_hs = INFINITY;  // approximate score of the winner
    uint32_t c0, c1;
    float h0, h1;
    while (next(&c0, &h0)) {
      if (!next(&c1, &h1)) {
        c1 = c0;
        h1 = h0;
      }
      const float ca0 = METRIC == vrs_exact::kCos ? cent_aux[c0] : 0.0f;
      const float ca1 = METRIC == vrs_exact::kCos ? cent_aux[c1] : 0.0f;
      float k0, k1;
      vrs_exact::lanes::rank_key2(METRIC, v, cent + (int64_t)c0 * dp, cent + (int64_t)c1 * dp, d, va, ca0, ca1, hl,
                                  mask, &k0, &k1);
      const bool b0 = hib ? (k0 > best_key || (k0 == best_key && (int)c0 < best))
                          : (k0 < best_key || (k0 == best_key && (int)c0 < best));
      if (b0) {
        best_key = k0;
        best = (int)c0;
        best_hs = h0;
      }
      const bool b1 = hib ? (k1 > best_key || (k1 == best_key && (int)c1 < best))
                          : (k1 < best_key || (k1 == best_key && (int)c1 < best));
      if (b1) {
        best_key = k1;
        best = (int)c1;
        best_hs = h1;
      }
    }
    if (hl == 0) {
      assign[i] = best;
      dist[i] = vrs_exact::finish(METRIC, best_key);
      if (pscore) pscore[i] = __fadd_ru(best_hs, 0.5f * absm);
    }
  }
}

// Exact distance of every point to its assigned centroid, in the reference's
// pair arithmetic (one half-warp per point), for the inertia of the last
// assignment step.
template <int METRIC>
__global__ void __launch_bounds__(128) kmeans_dist_kernel(const float* __restrict__ x, int64_t n, int d, int dp,
                                                          const float* __restrict__ cent,
                                                          const float* __restrict__ cent_aux,
                                                          const float* __restrict__ x_aux,
                                                          const int32_t* __restrict__ assign,
                                                          float* __restrict__ dist) {
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;
  if (i >= n) return;  // whole half-warps leave together
  const int hl = threadIdx.x & 15;
  const unsigned mask = 0xffffu << (threadIdx.x & 16);
  const int c = assign[i];
  const float va = METRIC == vrs_exact::kCos ? x_aux[i] : 0.0f;
  const float ca = METRIC == vrs_exact::kCos ? cent_aux[c] : 0.0f;
  const float key =
      vrs_exact::lanes::rank_key(METRIC, x + i * dp, cent + (int64_t)c * dp, d, va, ca, hl, mask);
  if (hl == 0) dist[i] = vrs_exact::finish(METRIC, key);
}

// Exact assignment of the flagged points (list F: flags[0] of them, indices
// from flags + 2): one CTA per point, its 16 half-warps split the centroids
// (half-warp h takes c = h, h + 16, ...), then the CTA keeps the best key,
// lowest centroid index on ties (kmeans.rs:361-407).
template <int METRIC>
__global__ void __launch_bounds__(256) kmeans_flagged_kernel(
    const float* __restrict__ x, int d, int dp, const float* __restrict__ cent,
    const float* __restrict__ cent_aux, const float* __restrict__ x_aux, int k, const int* __restrict__ flags,
    int32_t* __restrict__ assign, float* __restrict__ dist) {
  __shared__ float s_key[16];
  __shared__ int s_idx[16];
  const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
  const unsigned mask = 0xffffu << (threadIdx.x & 16);
  const bool hib = vrs_exact::higher_is_better(METRIC);
  const int count = flags[0];
  for (int f = blockIdx.x; f < count; f += gridDim.x) {
    const int64_t i = flags[2 + f];
    const float* v = x + i * dp;
    const float va = METRIC == vrs_exact::kCos ? x_aux[i] : 0.0f;
    int best = 0x7fffffff;
    float best_key = hib ? -INFINITY : INFINITY;
    for (int c = hw; c < k; c += 16) {
      const float ca = METRIC == vrs_exact::kCos ? cent_aux[c] : 0.0f;
      const float key = vrs_exact::lanes::rank_key(METRIC, v, cent + (int64_t)c * dp, d, va, ca, hl, mask);
      const bool better = hib ? (key > best_key) : (key < best_key);  // c increases: ties keep the lower
      if (better) {
        best_key = key;
        best = c;
      }
    }
    if (hl == 0) {
      s_key[hw] = best_key;
      s_idx[hw] = best;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bk = s_key[0];
      int bi = s_idx[0];
      for (int h = 1; h < 16; h++) {
        const float kk = s_key[h];
        const int ii = s_idx[h];
        const bool better = hib ? (kk > bk || (kk == bk && ii < bi)) : (kk < bk || (kk == bk && ii < bi));
        if (better) {
          bk = kk;
          bi = ii;
        }
      }
      assign[i] = bi;
      dist[i] = vrs_exact::finish(METRIC, bk);
    }
    __syncthreads();
  }
}

// Operand rows (bf16; cosine rows unit-normalised), |row|^2 and |row| for
// points or centroids; max |row| into *maxn; near-zero cosine rows flagged.
// One half-warp per row.
__global__ void __launch_bounds__(128) km_prep_rows_kernel(
    const float* __restrict__ x, int64_t n, int d, int dp, int metric, float op_scale, uint16_t* __restrict__ xb,
    float* __restrict__ sq, float* __restrict__ nrm, unsigned int* __restrict__ maxn,
    int* __restrict__ tiny_flag, int* __restrict__ any_tiny) {
  const int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 4;
  if (r >= n) return;
  const int hl = threadIdx.x & 15;
  const unsigned mask = 0xffffu << (threadIdx.x & 16);
  const int d16 = (d + 15) / 16 * 16;
  const float* v = x + r * dp;
  uint16_t* o = xb + r * d16;
  float scale = 1.0f;
  int tiny = 0;
  if (metric == vrs_exact::kCos) {
    const float s = sqrtf(vrs_exact::lanes::cos_dot(v, v, d, hl, mask));
    if (!(s >= 1e-4f)) {
      tiny = 1;
      scale = 0.0f;
    } else {
      scale = 1.0f / s;
    }
  }
  double ss = 0.0;
  for (int j = hl; j < d16; j += 16) {
    const float e = j < d ? v[j] : 0.0f;
    ss += (double)e * (double)e;
    o[j] = __half_as_ushort(__float2half_rn(metric == vrs_exact::kCos ? e * scale : e * op_scale));
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(mask, ss, off, 16);
  if (hl == 0) {
    if (sq) sq[r] = (float)ss;
    const float nr = (float)sqrt(ss);
    if (nrm) nrm[r] = nr;
    if (maxn) atomicMax(maxn, __float_as_uint(nr));
    if (tiny_flag) tiny_flag[r] = tiny;
    if (tiny && any_tiny) atomicOr(any_tiny, 1);
  }
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

int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int d16) {
  auto fn = encode_fn();
  if (!fn) {
    set_error(VRS_ERR_DRIVER, "cuTensorMapEncodeTiled unavailable");
    return VRS_ERR_DRIVER;
  }
  cuuint64_t dims[2] = {(cuuint64_t)d16, (cuuint64_t)std::max<int64_t>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)d16 * 2};
  cuuint32_t box[2] = {(cuuint32_t)KBW, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(VRS_ERR_DRIVER, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return VRS_ERR_DRIVER;
  }
  return VRS_OK;
}

template <int M>
int finalize_run(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
                 const float* x_aux, int k, const float* xq, const unsigned int* cmax, const Res* res,
                 void* groups, const int* force_full, int32_t* assign, float* dist, int* flags,
                 int num_sms, float inv_scale, float* pscore, cudaStream_t s) {
  const Groups gr = groups_at(groups, n);
  VRS_CUDA(cudaMemsetAsync(flags, 0, 2 * sizeof(int), s));
  kmeans_triage_kernel<M><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, d, xq, cmax, res, gr, force_full,
                                                                        assign, flags, inv_scale, pscore);
  VRS_CUDA(cudaGetLastError());
  // One resident wave (the kernel strides over the list): more blocks than
  // fit ran as a second wave with a tail.
  static const int multi_per_sm = [] {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kmeans_multi_kernel<M>, 128, 0) != cudaSuccess || b < 1)
      b = 4;
    return b;
  }();
  kmeans_multi_kernel<M><<<(unsigned)(num_sms * multi_per_sm), 128, 0, s>>>(x, n, d, dp, cent, cent_aux, x_aux, xq, cmax,
                                                                 res, gr, flags, assign, dist, inv_scale,
                                                                 pscore);
  VRS_CUDA(cudaGetLastError());
  kmeans_flagged_kernel<M><<<(unsigned)(num_sms * 8), 256, 0, s>>>(x, d, dp, cent, cent_aux, x_aux, k, flags,
                                                                   assign, dist);
  VRS_CUDA(cudaGetLastError());
  count_launch(3);
  return VRS_OK;
}

// Starting bound of the next Lloyd step (squared L2, Mahalanobis). Score
// units are |c|^2 - 2 x.c = |x - c|^2 - |x|^2. With c the point's centroid
// of the last step, pscore >= its score then and delta = |c_new - c_old|
// (the update's squared shift), |x - c_new| <= |x - c_old| + delta gives
// score_new(c) <= (sqrt(pscore + |x|^2) + delta)^2 - |x|^2; evaluated in
// f64 with a relative allowance for the f32 inputs (|x| and the shift are
// f32 results) and rounded up.
__global__ void kmeans_start_bound_kernel(int64_t n, const int32_t* __restrict__ assign,
                                          const float* __restrict__ pscore, const float* __restrict__ xq,
                                          const float* __restrict__ shift, float* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float ps = pscore[i];
  if (!(ps < INFINITY)) {
    out[i] = INFINITY;
    return;
  }
  const double x2 = (double)xq[i] * (double)xq[i];
  const double r = sqrt(fmax(0.0, ((double)ps + x2) * (1.0 + 1e-6)));
  const double dl = sqrt((double)shift[assign[i]] * (1.0 + 1e-4));
  const double ub = (r + dl) * (r + dl) - x2 * (1.0 - 1e-6) + 1e-5 * ((r + dl) * (r + dl) + x2) + 1e-30;
  out[i] = isfinite(ub) ? __double2float_ru(ub) : INFINITY;
}

}  // namespace

int start_bound(int64_t n, const int32_t* assign, const float* pscore, const float* xq, const float* shift,
                float* out, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  kmeans_start_bound_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, assign, pscore, xq, shift, out);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

bool supported(int metric, int d) {
  return d >= 1 && d <= 128 &&
         (metric == vrs_exact::kL2 || metric == vrs_exact::kMaha || metric == vrs_exact::kDot ||
          metric == vrs_exact::kCos);
}

int prep_rows(const float* x, int64_t n, int d, int dp, int metric, float op_scale, void* xb, float* sq,
              float* nrm, unsigned int* maxn, int* tiny_flag, int* any_tiny, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  km_prep_rows_kernel<<<(unsigned)((n * 16 + 127) / 128), 128, 0, s>>>(x, n, d, dp, metric, op_scale, (uint16_t*)xb,
                                                                      sq, nrm, maxn, tiny_flag, any_tiny);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int assign(const void* xb, int64_t n, const void* cb, int k, int d, const float* cn, const float* xq,
           const unsigned int* cmax, int metric, float op_scale, Res* res, void* groups, int* err, int num_sms,
           const float* init_bound, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  const int d16 = (d + 15) / 16 * 16;
  CUtensorMap tmA, tmB;
  VRS_TRY(make_tmap(&tmA, xb, n, d16));
  VRS_TRY(make_tmap(&tmB, cb, k, d16));
  AssignArgs a;
  a.cn = cn;
  a.xq = xq;
  a.cmax = cmax;
  a.n = n;
  a.k = k;
  a.d = d;
  a.ksteps = (d + 15) / 16;
  a.kblk = (d16 + KBW - 1) / KBW;
  a.mode = (metric == vrs_exact::kL2 || metric == vrs_exact::kMaha) ? 0 : 1;
  a.acc_scale = 1.0f / (op_scale * op_scale);
  a.inv_scale = 1.0f / op_scale;
  a.metric = metric;
  a.res = res;
  a.groups = groups_at(groups, n);
  a.err = err;
  a.init_bound = a.mode == 0 ? init_bound : nullptr;
  auto kern = a.mode == 0 ? kmeans_assign_tc_kernel<0> : kmeans_assign_tc_kernel<1>;
  VRS_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL));
  const int nptiles = (int)((n + BM * NACC - 1) / (BM * NACC));
  const int grid = std::max(1, std::min(nptiles, num_sms));
  kern<<<grid, THREADS, SMEM_TOTAL, s>>>(tmA, tmB, a);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int finalize(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
             const float* x_aux, int k, const float* xq, const unsigned int* cmax, int metric, const Res* res,
             void* groups, const int* force_full, int32_t* assign_out, float* dist, int* flags, int num_sms,
             float op_scale, float* pscore, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  switch (metric) {
    case vrs_exact::kL2:
      return finalize_run<vrs_exact::kL2>(x, n, d, dp, cent, cent_aux, x_aux, k, xq, cmax, res, groups, force_full,
                                          assign_out, dist, flags, num_sms, 1.0f / op_scale, pscore, s);
    case vrs_exact::kMaha:
      return finalize_run<vrs_exact::kMaha>(x, n, d, dp, cent, cent_aux, x_aux, k, xq, cmax, res, groups,
                                            force_full, assign_out, dist, flags, num_sms, 1.0f / op_scale, pscore,
                                            s);
    case vrs_exact::kDot:
      return finalize_run<vrs_exact::kDot>(x, n, d, dp, cent, cent_aux, x_aux, k, xq, cmax, res, groups,
                                           force_full, assign_out, dist, flags, num_sms, 1.0f / op_scale, nullptr,
                                           s);
    case vrs_exact::kCos:
      return finalize_run<vrs_exact::kCos>(x, n, d, dp, cent, cent_aux, x_aux, k, xq, cmax, res, groups,
                                           force_full, assign_out, dist, flags, num_sms, 1.0f / op_scale, nullptr,
                                           s);
  }
  set_error(VRS_ERR_INVALID_CONFIG, "k-means tensor-core finalize: unsupported metric");
  return VRS_ERR_INVALID_CONFIG;
}

int fill_dist(const float* x, int64_t n, int d, int dp, const float* cent, const float* cent_aux,
              const float* x_aux, int metric, const int32_t* assign, float* dist, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  const unsigned blocks = (unsigned)((n * 16 + 127) / 128);
  switch (metric) {
    case vrs_exact::kL2:
      kmeans_dist_kernel<vrs_exact::kL2><<<blocks, 128, 0, s>>>(x, n, d, dp, cent, cent_aux, x_aux, assign, dist);
      break;
    case vrs_exact::kMaha:
      kmeans_dist_kernel<vrs_exact::kMaha><<<blocks, 128, 0, s>>>(x, n, d, dp, cent, cent_aux, x_aux, assign, dist);
      break;
    case vrs_exact::kDot:
      kmeans_dist_kernel<vrs_exact::kDot><<<blocks, 128, 0, s>>>(x, n, d, dp, cent, cent_aux, x_aux, assign, dist);
      break;
    case vrs_exact::kCos:
      kmeans_dist_kernel<vrs_exact::kCos><<<blocks, 128, 0, s>>>(x, n, d, dp, cent, cent_aux, x_aux, assign, dist);
      break;
    default:
      set_error(VRS_ERR_INVALID_CONFIG, "k-means distance fill: unsupported metric");
      return VRS_ERR_INVALID_CONFIG;
  }
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

}  // namespace kmtc
}  // namespace vrs
