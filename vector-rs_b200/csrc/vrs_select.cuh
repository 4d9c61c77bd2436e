// vrs_select.cuh -- selection building blocks shared by the scan and
// select kernels: warp and block radix select of the k-th smallest score,
// in-place stream compaction, and a shared-memory bitonic sort, all on
// (score, id) candidates ordered by score then id.
#pragma once
#include "vrs_internal.cuh"

namespace vrs {
namespace sel {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ bool cand_less(const Cand& x, const Cand& y) {
  return x.hs < y.hs || (x.hs == y.hs && x.id < y.id);
}

__device__ __forceinline__ int warp_incl_scan(int v) {
  int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Given a 256-bin histogram in shared memory and a 1-based rank kk, one
// warp finds the digit holding the kk-th element and the count of elements
// in smaller digits. All 32 lanes return the same values.
__device__ __forceinline__ void warp_find_digit(const int* hist, int kk, int* digit, int* before) {
  int lane = threadIdx.x & 31;
  int local[8];
  int s = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    local[j] = hist[8 * lane + j];
    s += local[j];
  }
  int incl = warp_incl_scan(s);
  int excl = incl - s;
  unsigned m = __ballot_sync(kFull, excl < kk && kk <= incl);
  int src = m ? __ffs(m) - 1 : 31;
  int dg = 255, bf = 0;
  if (lane == src) {
    int acc = excl;
    dg = 8 * lane + 7;
    bf = acc;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      if (acc + local[j] >= kk) {
        dg = 8 * lane + j;
        bf = acc;
        break;
      }
      acc += local[j];
    }
  }
  *digit = __shfl_sync(kFull, dg, src);
  *before = __shfl_sync(kFull, bf, src);
}

// Warp radix select over a global-memory list. BY_ID = false: value =
// ord_key(hs) over all entries. BY_ID = true: value = id over the entries
// whose ord_key(hs) == match. Returns the kk-th smallest value (1-based)
// and, in *less, how many participating entries are strictly smaller.
template <bool BY_ID>
__device__ uint32_t warp_select(const Cand* list, int c, int kk, uint32_t match, int* hist,
                                int* less) {
  int lane = threadIdx.x & 31;
  uint32_t prefix = 0, pmask = 0;
  int below = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    for (int i = lane; i < c; i += 32) {
      Cand e = list[i];
      uint32_t hk = ord_key(e.hs);
      uint32_t v = BY_ID ? e.id : hk;
      bool part = BY_ID ? (hk == match) : true;
      if (part && (v & pmask) == prefix) atomicAdd(&hist[(v >> shift) & 255], 1);
    }
    __syncwarp();
    int digit, before;
    warp_find_digit(hist, kk, &digit, &before);
    kk -= before;
    below += before;
    prefix |= (uint32_t)digit << shift;
    pmask |= 0xffu << shift;
    __syncwarp();
  }
  *less = below;
  return prefix;
}

// In-place stream compaction of a warp-owned global list; returns the new count.
template <class Pred>
__device__ int warp_filter(Cand* list, int c, Pred keep_fn) {
  int lane = threadIdx.x & 31;
  int out = 0;
  for (int base = 0; base < c; base += 32) {
    int i = base + lane;
    Cand e;
    bool keep = false;
    if (i < c) {
      e = list[i];
      keep = keep_fn(e);
    }
    unsigned m = __ballot_sync(kFull, keep);
    if (keep) list[out + __popc(m & ((1u << lane) - 1))] = e;
    out += __popc(m);
  }
  __syncwarp();
  return out;
}

struct KeepExact {
  uint32_t kth, id_sel;
  __device__ bool operator()(const Cand& e) const {
    uint32_t k = ord_key(e.hs);
    return k < kth || (k == kth && e.id <= id_sel);
  }
};
struct KeepBound {
  float b;
  __device__ bool operator()(const Cand& e) const { return e.hs <= b; }
};

// Block-wide radix select over a shared-memory list (same contract as
// warp_select with BY_ID = false).
__device__ inline uint32_t block_select(const Cand* buf, int c, int kk, int* hist, int* s_res) {
  const int tid = threadIdx.x, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int i = tid; i < c; i += blockDim.x) {
      uint32_t v = ord_key(buf[i].hs);
      if ((v & pmask) == prefix) atomicAdd(&hist[(v >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
      int digit, before;
      warp_find_digit(hist, kk, &digit, &before);
      if (tid == 0) {
        s_res[0] = digit;
        s_res[1] = before;
      }
    }
    __syncthreads();
    kk -= s_res[1];
    prefix |= (uint32_t)s_res[0] << shift;
    pmask |= 0xffu << shift;
    __syncthreads();
  }
  return prefix;
}

// Block compaction of a shared list with a predicate; returns the new count.
template <class Pred>
__device__ int block_filter(Cand* buf, int c, Pred keep_fn, int* s_warp_tot) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  int out = 0;
  for (int base = 0; base < c; base += blockDim.x) {
    int i = base + tid;
    Cand e;
    bool keep = false;
    if (i < c) {
      e = buf[i];
      keep = keep_fn(e);
    }
    unsigned m = __ballot_sync(kFull, keep);
    if (lane == 0) s_warp_tot[warp] = __popc(m);
    __syncthreads();
    int woff = 0, tot = 0;
    for (int w = 0; w < nw; w++) {
      if (w < warp) woff += s_warp_tot[w];
      tot += s_warp_tot[w];
    }
    __syncthreads();
    if (keep) buf[out + woff + __popc(m & ((1u << lane) - 1))] = e;
    out += tot;
    __syncthreads();
  }
  return out;
}

__device__ inline void block_bitonic_sort(Cand* s, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        int ixj = i ^ j;
        if (ixj > i) {
          bool asc = (i & k) == 0;
          Cand x = s[i], y = s[ixj];
          if (cand_less(y, x) == asc) {
            s[i] = y;
            s[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}


}  // namespace sel
}  // namespace vrs
