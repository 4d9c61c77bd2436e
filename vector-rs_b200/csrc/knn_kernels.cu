// knn_kernels.cu -- CUDA-core kernels of the flat kNN path:
//   * knn_scan_exact: streams the shard, scores (query, row) pairs in the
//     reference's exact arithmetic order, and keeps per-(segment, query)
//     candidate lists bounded by a running k-th best (radix-select
//     compaction); the Q x N score matrix never reaches HBM;
//   * knn_select: per query, gathers the segment lists, selects the k-th
//     best, re-ranks the survivors exactly and sorts by (score, id);
//   * merge_pairs: G-way merge of per-rank top-k lists after the NCCL
//     all-gather (replaces CollectiveOps::top_k_reduce,
//     crates/vector-cuda/src/ddp/collective.rs:115-159);
//   * small layout kernels (row padding, Hellinger roots, cosine norms).
// Reference kernels these replace: knn_compute_distance_matrix and
// knn_topk_select, crates/vector-cuda/src/kernels/knn.cu:21-305.
#include <float.h>

#include "vrs_exact.cuh"
#include "vrs_exact_lanes.cuh"
#include "vrs_internal.cuh"
#include "vrs_select.cuh"

namespace vrs {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanQT = 32;  // query slots per CTA
constexpr int kScanNT = 64;  // rows per tile
using namespace sel;

// Shrinks one (segment, query) list once it is nearly full. Exact scores
// keep exactly the k best by (score, id); approximate scores keep every
// entry within the acceptance bound of the k-th best (and flag overflow when
// near-ties leave no room).
__device__ void warp_compact(const KnnScanArgs& a, Cand* list, int c, float absm, int* hist,
                             int* new_c, float* new_bound, bool* ovf) {
  int less;
  uint32_t kth = warp_select<false>(list, c, a.k, 0, hist, &less);
  float tau = ord_inv(kth);
  if (a.kind == kExactScores) {
    int less2;
    uint32_t id_sel = warp_select<true>(list, c, a.k - less, kth, hist, &less2);
    *new_c = warp_filter(list, c, KeepExact{kth, id_sel});
    *new_bound = tau;
    *ovf = false;
  } else {
    float b = accept_bound(a.kind, tau, a.rho, absm);
    *new_c = warp_filter(list, c, KeepBound{b});
    *new_bound = b;
    *ovf = *new_c > a.cap - kScanNT;
  }
}

template <int METRIC>
__device__ __forceinline__ float pair_key(const float* q, const float* x, int d, float qa, float xa) {
  return vrs_exact::rank_key(METRIC, q, x, d, qa, xa);
}

template <int METRIC>
__global__ void __launch_bounds__(kScanThreads) knn_scan_exact_kernel(KnnScanArgs a) {
  __shared__ float s_bound[kScanQT];
  __shared__ int s_cnt[kScanQT];
  __shared__ int s_hist[kScanThreads / 32][256];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int qt0 = blockIdx.x * kScanQT;
  const int seg = blockIdx.y;
  const int64_t row_begin = (int64_t)seg * a.seg_len;
  const int64_t row_end = min(a.n, row_begin + a.seg_len);
  if (tid < kScanQT) {
    s_bound[tid] = INFINITY;
    s_cnt[tid] = 0;
  }
  __syncthreads();
  const int qs = tid >> 3;
  const int slot = qt0 + qs;
  const bool valid = slot < a.nq;
  const int qrow = valid ? (a.q_index ? a.q_index[slot] : slot) : 0;
  const float* qp = a.q + (int64_t)qrow * a.dp;
  const float qa = (METRIC == vrs_exact::kCos && valid) ? a.q_aux[qrow] : 0.0f;
  Cand* list = a.cand + ((int64_t)seg * a.nq + (valid ? slot : 0)) * a.cap;

  for (int64_t t0 = row_begin; t0 < row_end; t0 += kScanNT) {
    const float bound = s_bound[qs];
#pragma unroll 1
    for (int j = 0; j < kScanNT / 8; j++) {
      const int64_t row = t0 + (tid & 7) + 8 * j;
      if (valid && row < row_end) {
        const float* xp = a.base + row * a.dp;
        const float xa = (METRIC == vrs_exact::kCos) ? a.base_aux[row] : 0.0f;
        const float key = pair_key<METRIC>(qp, xp, a.d, qa, xa);
        const float hs = vrs_exact::heap_score(METRIC, key);
        if (hs < bound) {
          int pos = atomicAdd(&s_cnt[qs], 1);
          list[pos] = Cand{hs, (uint32_t)row};
        }
      }
    }
    __syncthreads();
    for (int s = warp; s < kScanQT; s += kScanThreads / 32) {
      int c = s_cnt[s];
      if (qt0 + s < a.nq && c > a.cap - kScanNT) {
        Cand* l = a.cand + ((int64_t)seg * a.nq + qt0 + s) * a.cap;
        int nc;
        float nb;
        bool ovf;
        warp_compact(a, l, c, 0.0f, s_hist[warp], &nc, &nb, &ovf);
        if ((threadIdx.x & 31) == 0) {
          s_cnt[s] = nc;
          s_bound[s] = nb;
        }
      }
    }
    __syncthreads();
  }
  // Final compaction so the select step sees at most ~k entries per segment.
  for (int s = warp; s < kScanQT; s += kScanThreads / 32) {
    int c = s_cnt[s];
    if (qt0 + s < a.nq && c > a.k) {
      Cand* l = a.cand + ((int64_t)seg * a.nq + qt0 + s) * a.cap;
      int nc;
      float nb;
      bool ovf;
      warp_compact(a, l, c, 0.0f, s_hist[warp], &nc, &nb, &ovf);
      if ((threadIdx.x & 31) == 0) s_cnt[s] = nc;
    }
  }
  __syncthreads();
  if (tid < kScanQT && qt0 + tid < a.nq) a.cnt[(int64_t)seg * a.nq + qt0 + tid] = s_cnt[tid];
}

// ------------------------------------------------------------------ select
// Certified limit of a slot whose bound could not be checked alone, in
// exact heap-score units: no unkept row of this shard scores below it. The
// scan kept every row whose approximate score is within sb, and absm / 2
// covers the approximate score's error plus the exact score's rounding, so
// an unkept row's exact score exceeds sb - absm / 2 (plus |q|^2 for the
// squared-L2 scores, which leave it out); both steps round down.
__device__ __forceinline__ float certified_limit(const KnnSelectArgs& a, float sb, int qrow) {
  const float lim = __fsub_rd(sb, 0.5f * a.absm[qrow]);
  return a.q_sq ? __fadd_rd(lim, a.q_sq[qrow]) : lim;
}

template <int METRIC>
__device__ void select_one(const KnnSelectArgs& a, int slot, Cand* sbuf, int* s_hist, int* s_res, int* s_wt,
                           int* s_off) {
  const int tid = threadIdx.x;
  const int qrow = a.q_index ? a.q_index[slot] : slot;
  if (tid == 0) {
    int tot = 0;
    for (int s = 0; s < a.nseg; s++) {
      s_off[s] = tot;
      tot += a.cnt[(int64_t)s * a.nq + slot];
    }
    s_off[a.nseg] = tot;
  }
  __syncthreads();
  int total = s_off[a.nseg];
  if (total > a.max_sort) {
    if (tid == 0) a.overflow[slot] = 1;
    return;
  }
  for (int s = 0; s < a.nseg; s++) {
    const Cand* l = a.cand + ((int64_t)s * a.nq + slot) * a.cap;
    int c = s_off[s + 1] - s_off[s];
    for (int i = tid; i < c; i += blockDim.x) sbuf[s_off[s] + i] = l[i];
  }
  __syncthreads();
  // k-th best scan score over all segments -> acceptance bound -> survivors.
  int R = total;
  const float sb = a.init_bound ? a.init_bound[slot] : INFINITY;
  bool cut = false;  // unverified bound, merge pairs cut at `lim`
  if (total > a.k || (total == a.k && sb < INFINITY)) {
    uint32_t kth = block_select(sbuf, total, a.k, s_hist, s_res);
    float tau = ord_inv(kth);
    float absm = a.kind == kAbsMargin ? a.absm[qrow] : 0.0f;
    float b = accept_bound(a.kind, tau, a.rho, absm);
    if (!(b <= sb)) {
      if (!a.certify) {
        if (tid == 0) a.overflow[slot] = 1;
        return;
      }
      cut = true;  // b > sb keeps every stored row
    }
    R = block_filter(sbuf, total, KeepBound{b}, s_wt);
  } else if (total < a.k && sb < INFINITY) {
    if (!a.certify) {
      if (tid == 0) a.overflow[slot] = 1;
      return;
    }
    cut = true;
  }
  const float lim = cut ? certified_limit(a, sb, qrow) : INFINITY;
  // Exact re-rank of approximate survivors in the reference's order.
  if (a.kind != kExactScores) {
    const float* qp = a.q + (int64_t)qrow * a.dp;
    const float qa = METRIC == vrs_exact::kCos ? a.q_aux[qrow] : 0.0f;
    for (int i = tid; i < R; i += blockDim.x) {
      uint32_t row = sbuf[i].id;
      const float xa = METRIC == vrs_exact::kCos ? a.base_aux[row] : 0.0f;
      float key = vrs_exact::rank_key(METRIC, qp, a.base + (int64_t)row * a.dp, a.d, qa, xa);
      sbuf[i].hs = vrs_exact::heap_score(METRIC, key);
    }
    __syncthreads();
  }
  // Rows whose approximate score carries no error bound are always re-ranked.
  if (a.n_tiny > 0) {
    if (R + a.n_tiny > a.max_sort) {
      if (tid == 0) a.overflow[slot] = 1;
      return;
    }
    const float* qp = a.q + (int64_t)qrow * a.dp;
    const float qa = METRIC == vrs_exact::kCos ? a.q_aux[qrow] : 0.0f;
    for (int i = tid; i < a.n_tiny; i += blockDim.x) {
      uint32_t row = a.tiny[i];
      const float xa = METRIC == vrs_exact::kCos ? a.base_aux[row] : 0.0f;
      float key = vrs_exact::rank_key(METRIC, qp, a.base + (int64_t)row * a.dp, a.d, qa, xa);
      sbuf[R + i] = Cand{vrs_exact::heap_score(METRIC, key), row};
    }
    R += a.n_tiny;
    __syncthreads();
  }
  int P = 1;
  while (P < R) P <<= 1;
  if (P > a.max_sort) {
    if (tid == 0) a.overflow[slot] = 1;
    return;
  }
  for (int i = R + tid; i < P; i += blockDim.x) sbuf[i] = Cand{INFINITY, 0xffffffffu};
  __syncthreads();
  block_bitonic_sort(sbuf, P);
  for (int r = tid; r < a.k; r += blockDim.x) {
    Cand e = r < R ? sbuf[r] : Cand{INFINITY, 0xffffffffu};
    uint32_t gid = e.id == 0xffffffffu ? 0xffffffffu : e.id + a.id_offset;
    if (cut && !(e.hs < lim)) {
      // Sorted: rows below lim form a prefix; the sentinel follows it.
      const bool first = r == 0 || (r - 1 < R && sbuf[r - 1].hs < lim);
      e = first ? Cand{lim, kSentinelId} : Cand{INFINITY, 0xffffffffu};
      gid = e.id;
    }
    if (a.out_pairs) a.out_pairs[(int64_t)qrow * a.k + r] = Cand{e.hs, gid};
    if (a.out_dist) {
      float key = vrs_exact::higher_is_better(METRIC) ? -e.hs : e.hs;
      a.out_dist[(int64_t)qrow * a.k + r] = e.id == 0xffffffffu ? NAN : vrs_exact::finish(METRIC, key);
      a.out_id[(int64_t)qrow * a.k + r] = gid;
    }
  }
}

// Block per query (grid = nq), or, with a.retry, a small grid striding over
// the queries and taking only those the warp select flagged (2).
template <int METRIC>
__global__ void __launch_bounds__(256) knn_select_kernel(KnnSelectArgs a) {
  extern __shared__ Cand sbuf[];
  __shared__ int s_hist[256];
  __shared__ int s_res[4];
  __shared__ int s_wt[32];
  __shared__ int s_off[65];
  if (!a.retry) {
    if (a.overflow[blockIdx.x]) return;
    select_one<METRIC>(a, blockIdx.x, sbuf, s_hist, s_res, s_wt, s_off);
    return;
  }
  for (int slot = blockIdx.x; slot < a.nq; slot += gridDim.x) {
    if (a.overflow[slot] != 2) continue;  // uniform over the block
    __syncthreads();
    if (threadIdx.x == 0) a.overflow[slot] = 0;
    __syncthreads();
    select_one<METRIC>(a, slot, sbuf, s_hist, s_res, s_wt, s_off);
    __syncthreads();
  }
}

// ------------------------------------------------ select, warp per query
// For approximate scans (tensor-core path): one warp per query. The k-th
// best approximate score over the segment lists is found by a warp radix
// select reading the lists in place; survivors within the acceptance bound
// are copied to shared memory, re-ranked exactly by half-warps (the 16 lanes
// are the reference's 16 SIMD lanes, loads coalesced), sorted by
// (score, id) with a warp bitonic sort, and written out.
constexpr int kSelWarps = 4;
constexpr int kSelRmax = 1024;

template <int METRIC>
__global__ void __launch_bounds__(kSelWarps * 32) knn_select_warp_kernel(KnnSelectArgs a) {
  __shared__ int s_hist[kSelWarps][256];
  __shared__ Cand s_buf[kSelWarps][kSelRmax];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = blockIdx.x * kSelWarps + warp;
  if (slot >= a.nq) return;
  if (a.overflow[slot]) return;
  const int qrow = a.q_index ? a.q_index[slot] : slot;
  Cand* buf = s_buf[warp];
  int* hist = s_hist[warp];
  // Lane l owns list l: its count and the exclusive prefix of the counts,
  // so the lists read as one flattened array of `total` entries.
  const int cnt_l = lane < a.nseg ? a.cnt[(int64_t)lane * a.nq + slot] : 0;
  const int pre_l = warp_incl_scan(cnt_l) - cnt_l;
  const int total = __shfl_sync(kFull, pre_l + cnt_l, 31);
  // Entry j of the flattened lists (all lanes call together; j may be out
  // of range, in which case nothing is read).
  auto entry = [&](int j, bool* valid) -> Cand {
    int lo = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
      const int pm = __shfl_sync(kFull, pre_l, lo + step);
      if (lo + step < a.nseg && pm <= j) lo += step;
    }
    const int p0 = __shfl_sync(kFull, pre_l, lo);
    *valid = j < total;
    Cand e{INFINITY, 0xffffffffu};
    if (*valid) e = a.cand[((int64_t)lo * a.nq + slot) * a.cap + (j - p0)];
    return e;
  };
  constexpr int kBatch = 4;  // entries per lane in flight

  float bound = INFINITY;
  const float sb = a.init_bound ? a.init_bound[slot] : INFINITY;
  bool cut = false;  // unverified bound, merge pairs cut at `lim`
  if (total < a.k && sb < INFINITY) {
    // Fewer than k rows within an unproven bound.
    if (!a.certify) {
      if (lane == 0) a.overflow[slot] = 1;
      return;
    }
    cut = true;
  }
  if (total > a.k || (total == a.k && sb < INFINITY)) {
    uint32_t prefix = 0, pmask = 0;
    int kk = a.k;
    // Up to kSelRmax * 2 keys are staged in shared memory (the candidate
    // buffer, free until the compaction below), so the radix passes read
    // global memory once; longer lists are read once per pass.
    uint32_t* keys = reinterpret_cast<uint32_t*>(buf);
    const bool staged = total <= 2 * kSelRmax;
    if (staged) {
      for (int j0 = 0; j0 < total; j0 += 32 * kBatch) {
        Cand e[kBatch];
        bool v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; u++) e[u] = entry(j0 + u * 32 + lane, &v[u]);
#pragma unroll
        for (int u = 0; u < kBatch; u++)
          if (v[u]) keys[j0 + u * 32 + lane] = ord_key(e[u].hs);
      }
      __syncwarp();
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = lane; b < 256; b += 32) hist[b] = 0;
      __syncwarp();
      if (staged) {
        for (int i = lane; i < total; i += 32) {
          const uint32_t v = keys[i];
          if ((v & pmask) == prefix) atomicAdd(&hist[(v >> shift) & 255], 1);
        }
      } else {
        for (int sgm = 0; sgm < a.nseg; sgm++) {
          const int cs = __shfl_sync(kFull, cnt_l, sgm);
          const Cand* l = a.cand + ((int64_t)sgm * a.nq + slot) * a.cap;
          for (int i = lane; i < cs; i += 32) {
            const uint32_t v = ord_key(l[i].hs);
            if ((v & pmask) == prefix) atomicAdd(&hist[(v >> shift) & 255], 1);
          }
        }
      }
      __syncwarp();
      int digit, before;
      warp_find_digit(hist, kk, &digit, &before);
      kk -= before;
      prefix |= (uint32_t)digit << shift;
      pmask |= 0xffu << shift;
      __syncwarp();
    }
    const float absm = a.kind == kAbsMargin ? a.absm[qrow] : 0.0f;
    bound = accept_bound(a.kind, ord_inv(prefix), a.rho, absm);
    if (!(bound <= sb)) {
      // The scan's bound may have cut a top-k row (bound > sb keeps every
      // stored row).
      if (!a.certify) {
        if (lane == 0) a.overflow[slot] = 1;
        return;
      }
      cut = true;
    }
  }
  const float lim = cut ? certified_limit(a, sb, qrow) : INFINITY;
  // Survivors -> shared memory (batched reads of the flattened lists).
  int R = 0;
  for (int j0 = 0; j0 < total; j0 += 32 * kBatch) {
    Cand e[kBatch];
    bool v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; u++) e[u] = entry(j0 + u * 32 + lane, &v[u]);
#pragma unroll
    for (int u = 0; u < kBatch; u++) {
      const bool keep = v[u] && e[u].hs <= bound;
      const unsigned m = __ballot_sync(kFull, keep);
      const int pos = R + __popc(m & ((1u << lane) - 1));
      if (keep && pos < kSelRmax) buf[pos] = e[u];
      R += __popc(m);
    }
  }
  if (R + a.n_tiny > kSelRmax) {
    if (lane == 0) a.overflow[slot] = 2;  // retried by the block select (knn_select_kernel, retry)
    return;
  }
  __syncwarp();
  // Exact re-rank, four candidates per warp step (two per half-warp, both
  // rows' loads in flight); rows without an error bound (near-zero cosine
  // rows) are scored here too.
  const float* qp = a.q + (int64_t)qrow * a.dp;
  const float qa = METRIC == vrs_exact::kCos ? a.q_aux[qrow] : 0.0f;
  const int half = lane >> 4, hl = lane & 15;
  const int RT = R + a.n_tiny;
  // Rows of step it + 1 -> L2 while step it is scored (16 lanes, one 128-byte
  // line each: four rows of up to four lines; longer rows are fetched as
  // they are read).
  auto prefetch_step = [&](int it) {
    const int i = 4 * it + (lane >> 2);
    if (lane < 16 && i < RT && (lane & 3) * 32 < a.d) {
      const uint32_t row = i < R ? buf[i].id : a.tiny[i - R];
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a.base + (int64_t)row * a.dp + (lane & 3) * 32));
    }
  };
  prefetch_step(0);
  for (int it = 0; 4 * it < RT; it++) {
    prefetch_step(it + 1);
    const int i0 = 4 * it + half, i1 = 4 * it + 2 + half;
    const bool act0 = i0 < RT, act1 = i1 < RT;
    const int ii0 = act0 ? i0 : 4 * it, ii1 = act1 ? i1 : 4 * it;
    const uint32_t row0 = ii0 < R ? buf[ii0].id : a.tiny[ii0 - R];
    const uint32_t row1 = ii1 < R ? buf[ii1].id : a.tiny[ii1 - R];
    const float xa0 = METRIC == vrs_exact::kCos ? a.base_aux[row0] : 0.0f;
    const float xa1 = METRIC == vrs_exact::kCos ? a.base_aux[row1] : 0.0f;
    float key0, key1;
    vrs_exact::lanes::rank_key2(METRIC, qp, a.base + (int64_t)row0 * a.dp, a.base + (int64_t)row1 * a.dp,
                                a.d, qa, xa0, xa1, hl, kFull, &key0, &key1);
    __syncwarp();
    if (hl == 0) {
      if (act0) buf[i0] = Cand{vrs_exact::heap_score(METRIC, key0), row0};
      if (act1) buf[i1] = Cand{vrs_exact::heap_score(METRIC, key1), row1};
    }
  }
  __syncwarp();
  int P = 32;
  while (P < RT) P <<= 1;
  for (int i = RT + lane; i < P; i += 32) buf[i] = Cand{INFINITY, 0xffffffffu};
  __syncwarp();
  for (int kb = 2; kb <= P; kb <<= 1) {
    for (int j = kb >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < P; i += 32) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const bool asc = (i & kb) == 0;
          const Cand x = buf[i], y = buf[ixj];
          if (cand_less(y, x) == asc) {
            buf[i] = y;
            buf[ixj] = x;
          }
        }
      }
      __syncwarp();
    }
  }
  for (int r = lane; r < a.k; r += 32) {
    Cand e = r < RT ? buf[r] : Cand{INFINITY, 0xffffffffu};
    uint32_t gid = e.id == 0xffffffffu ? 0xffffffffu : e.id + a.id_offset;
    if (cut && !(e.hs < lim)) {
      // Sorted: rows below lim form a prefix; the sentinel follows it.
      const bool first = r == 0 || (r - 1 < RT && buf[r - 1].hs < lim);
      e = first ? Cand{lim, kSentinelId} : Cand{INFINITY, 0xffffffffu};
      gid = e.id;
    }
    if (a.out_pairs) a.out_pairs[(int64_t)qrow * a.k + r] = Cand{e.hs, gid};
    if (a.out_dist) {
      const float key = vrs_exact::higher_is_better(METRIC) ? -e.hs : e.hs;
      a.out_dist[(int64_t)qrow * a.k + r] = e.id == 0xffffffffu ? NAN : vrs_exact::finish(METRIC, key);
      a.out_id[(int64_t)qrow * a.k + r] = gid;
    }
  }
}

// --------------------------------------------------------------- merge
template <int METRIC>
__global__ void __launch_bounds__(256) merge_pairs_kernel(const Cand* g, int nlists, int nq, int k,
                                                           float* out_dist, uint32_t* out_id, int* flags) {
  extern __shared__ Cand sbuf[];
  const int q = blockIdx.x;
  const int T = nlists * k;
  int P = 1;
  while (P < T) P <<= 1;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    if (i < T) {
      int l = i / k, r = i % k;
      sbuf[i] = g[((int64_t)l * nq + q) * k + r];
    } else {
      sbuf[i] = Cand{INFINITY, 0xffffffffu};
    }
  }
  __syncthreads();
  block_bitonic_sort(sbuf, P);
  for (int r = threadIdx.x; r < k; r += blockDim.x) {
    Cand e = sbuf[r];
    if (flags && e.id == kSentinelId) flags[q] = 1;
    float key = vrs_exact::higher_is_better(METRIC) ? -e.hs : e.hs;
    out_dist[(int64_t)q * k + r] = e.id == 0xffffffffu ? NAN : vrs_exact::finish(METRIC, key);
    out_id[(int64_t)q * k + r] = e.id;
  }
}

// G-way merge of lists that are each sorted by (score, id) (every rank's
// select writes its top-k' sorted): an element's output position is its
// index in its own list plus, for every other list, the number of elements
// ordered before it, found by binary search. The order is (score, id, list),
// so padding entries (+inf, 0xffffffff) of different lists stay distinct and
// exactly k' elements land below k'. No sort.
template <int METRIC>
__global__ void __launch_bounds__(256) merge_sorted_kernel(const Cand* g, int nlists, int nq, int k,
                                                           float* out_dist, uint32_t* out_id, int* flags) {
  extern __shared__ Cand sl[];  // [nlists][k]
  const int q = blockIdx.x;
  const int T = nlists * k;
  for (int i = threadIdx.x; i < T; i += blockDim.x) {
    const int l = i / k, r = i - l * k;
    sl[i] = g[((int64_t)l * nq + q) * k + r];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < T; i += blockDim.x) {
    const int l = i / k, j = i - l * k;
    const Cand e = sl[i];
    int rank = j;
    for (int m = 0; m < nlists && rank < k; m++) {
      if (m == l) continue;
      const Cand* lm = sl + m * k;
      int lo = 0, hi = k;  // first position of list m not ordered before e
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const Cand c = lm[mid];
        const bool before = cand_less(c, e) || (!cand_less(e, c) && m < l);
        if (before) lo = mid + 1;
        else hi = mid;
      }
      rank += lo;
    }
    if (rank < k) {
      if (flags && e.id == kSentinelId) flags[q] = 1;
      const float key = vrs_exact::higher_is_better(METRIC) ? -e.hs : e.hs;
      out_dist[(int64_t)q * k + rank] = e.id == 0xffffffffu ? NAN : vrs_exact::finish(METRIC, key);
      out_id[(int64_t)q * k + rank] = e.id;
    }
  }
}

__global__ void flag_pairs_kernel(const int* __restrict__ overflow, int nq, int k, Cand* __restrict__ pairs) {
  const int q = blockIdx.x;
  if (q >= nq || !overflow[q]) return;
  for (int r = threadIdx.x; r < k; r += blockDim.x)
    pairs[(int64_t)q * k + r] = r == 0 ? Cand{-INFINITY, kSentinelId} : Cand{INFINITY, 0xffffffffu};
}

__global__ void scatter_flags_kernel(const int* __restrict__ src, const int* __restrict__ idx, int n,
                                     int* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[idx[i]] = src[i];
}

template <int METRIC>
__global__ void finish_pairs_kernel(const Cand* p, int64_t count, float* out_dist, uint32_t* out_id) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= count) return;
  Cand e = p[i];
  float key = vrs_exact::higher_is_better(METRIC) ? -e.hs : e.hs;
  out_dist[i] = e.id == 0xffffffffu ? NAN : vrs_exact::finish(METRIC, key);
  out_id[i] = e.id;
}

// ------------------------------------------------------------- layout
__global__ void pad_rows_kernel(const float* __restrict__ src, int64_t rows, int d, int dp,
                                float* __restrict__ dst, int transform) {
  int64_t total = rows * dp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / dp;
    int c = (int)(i - r * dp);
    float v = c < d ? src[r * d + c] : 0.0f;
    if (transform == 1) v = vrs_exact::root_abs(v);
    dst[i] = v;
  }
}

__global__ void cos_norms_kernel(const float* __restrict__ x, int64_t rows, int d, int dp,
                                 float* __restrict__ out) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r < rows) out[r] = vrs_exact::cos_norm_sq(x + r * dp, d);
}

template <template <int> class F, class... Args>
int dispatch_metric(int metric, Args... args) {
  switch (metric) {
    case 0: return F<0>::run(args...);
    case 1: return F<1>::run(args...);
    case 2: return F<2>::run(args...);
    case 3: return F<3>::run(args...);
    case 4: return F<4>::run(args...);
    case 5: return F<5>::run(args...);
    case 6: return F<6>::run(args...);
    case 7: return F<7>::run(args...);
    case 8: return F<8>::run(args...);
    case 9: return F<9>::run(args...);
  }
  set_error(VRS_ERR_INVALID_CONFIG, "unknown metric code " + std::to_string(metric));
  return VRS_ERR_INVALID_CONFIG;
}

template <int M>
struct ScanExactL {
  static int run(const KnnScanArgs& a, cudaStream_t s) {
    dim3 grid((a.nq + kScanQT - 1) / kScanQT, a.nseg);
    knn_scan_exact_kernel<M><<<grid, kScanThreads, 0, s>>>(a);
    VRS_CUDA(cudaGetLastError());
    count_launch();
    return VRS_OK;
  }
};

template <int M>
struct SelectL {
  static int run(const KnnSelectArgs& a, cudaStream_t s) {
    size_t smem = (size_t)a.max_sort * sizeof(Cand);
    VRS_CUDA(cudaFuncSetAttribute(knn_select_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    const unsigned grid = a.retry ? (unsigned)std::min(a.nq, 148 * 2) : (unsigned)a.nq;
    knn_select_kernel<M><<<grid, 256, smem, s>>>(a);
    VRS_CUDA(cudaGetLastError());
    count_launch();
    return VRS_OK;
  }
};

template <int M>
struct SelectWarpL {
  static int run(const KnnSelectArgs& a, cudaStream_t s) {
    if (M != vrs_exact::kL2 && M != vrs_exact::kMaha && M != vrs_exact::kDot && M != vrs_exact::kCos) {
      set_error(VRS_ERR_INVALID_CONFIG, "warp select supports L2/Mahalanobis/dot/cosine");
      return VRS_ERR_INVALID_CONFIG;
    }
    if (a.nseg > 32 || a.k > kSelRmax) {
      set_error(VRS_ERR_INVALID_CONFIG, "warp select needs nseg <= 32 and k <= 512");
      return VRS_ERR_INVALID_CONFIG;
    }
    knn_select_warp_kernel<M><<<(a.nq + kSelWarps - 1) / kSelWarps, kSelWarps * 32, 0, s>>>(a);
    VRS_CUDA(cudaGetLastError());
    count_launch();
    return VRS_OK;
  }
};

template <int M>
struct MergeL {
  static int run(const Cand* g, int nlists, int nq, int k, float* od, uint32_t* oi, int* flags, cudaStream_t s) {
    const size_t lsm = (size_t)nlists * k * sizeof(Cand);
    if (lsm <= 200 * 1024) {
      VRS_CUDA(cudaFuncSetAttribute(merge_sorted_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsm));
      merge_sorted_kernel<M><<<nq, 256, lsm, s>>>(g, nlists, nq, k, od, oi, flags);
      VRS_CUDA(cudaGetLastError());
      count_launch();
      return VRS_OK;
    }
    int P = 1;
    while (P < nlists * k) P <<= 1;
    size_t smem = (size_t)P * sizeof(Cand);
    VRS_CUDA(cudaFuncSetAttribute(merge_pairs_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    merge_pairs_kernel<M><<<nq, 256, smem, s>>>(g, nlists, nq, k, od, oi, flags);
    VRS_CUDA(cudaGetLastError());
    count_launch();
    return VRS_OK;
  }
};

template <int M>
struct FinishL {
  static int run(const Cand* p, int64_t count, float* od, uint32_t* oi, cudaStream_t s) {
    if (count == 0) return VRS_OK;
    finish_pairs_kernel<M><<<(unsigned)((count + 255) / 256), 256, 0, s>>>(p, count, od, oi);
    VRS_CUDA(cudaGetLastError());
    count_launch();
    return VRS_OK;
  }
};

}  // namespace

int launch_knn_scan_exact(const KnnScanArgs& a, cudaStream_t s) {
  if (a.nq == 0 || a.n == 0) return VRS_OK;
  return dispatch_metric<ScanExactL>(a.metric, a, s);
}

int launch_knn_select(const KnnSelectArgs& a, cudaStream_t s) {
  if (a.nq == 0) return VRS_OK;
  return dispatch_metric<SelectL>(a.metric, a, s);
}

int launch_knn_select_warp(const KnnSelectArgs& a, cudaStream_t s) {
  if (a.nq == 0) return VRS_OK;
  return dispatch_metric<SelectWarpL>(a.metric, a, s);
}

int launch_merge_pairs(const Cand* gathered, int nlists, int nq, int k, int metric, float* out_dist,
                       uint32_t* out_id, int* flags, cudaStream_t s) {
  if (nq == 0 || k == 0) return VRS_OK;
  return dispatch_metric<MergeL>(metric, gathered, nlists, nq, k, out_dist, out_id, flags, s);
}

int launch_scatter_flags(const int* src, const int* idx, int n, int* dst, cudaStream_t s) {
  if (n == 0) return VRS_OK;
  scatter_flags_kernel<<<(n + 255) / 256, 256, 0, s>>>(src, idx, n, dst);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int launch_flag_pairs(const int* overflow, int nq, int k, Cand* pairs, cudaStream_t s) {
  if (nq == 0 || k == 0) return VRS_OK;
  flag_pairs_kernel<<<nq, 128, 0, s>>>(overflow, nq, k, pairs);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int launch_finish_pairs(const Cand* pairs, int64_t count, int metric, float* out_dist,
                        uint32_t* out_id, cudaStream_t s) {
  return dispatch_metric<FinishL>(metric, pairs, count, out_dist, out_id, s);
}

int launch_pad_rows(const float* src, int64_t rows, int d, int dp, float* dst, int transform,
                    cudaStream_t s) {
  if (rows == 0) return VRS_OK;
  int64_t total = rows * dp;
  int64_t nblk = (total + 255) / 256;
  unsigned blocks = (unsigned)(nblk < 148 * 64 ? nblk : 148 * 64);
  pad_rows_kernel<<<blocks, 256, 0, s>>>(src, rows, d, dp, dst, transform);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

int launch_cos_norms(const float* x, int64_t rows, int d, int dp, float* out, cudaStream_t s) {
  if (rows == 0) return VRS_OK;
  cos_norms_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, s>>>(x, rows, d, dp, out);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

}  // namespace vrs
