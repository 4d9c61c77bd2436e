// ivfpq.cu -- IVF-PQ search with asymmetric distance computation (ADC) on
// the GPU: IvfPqIndex::search_with_nprobe
// (crates/vector-index/src/ivf/mod.rs:265-345) over a trained index, with
// ProductQuantizer::compute_adc_lut and compute_distance_with_lut
// (crates/vector-index/src/ivf/pq.rs:233-296).
//
// Per query the reference
//   1. ranks the coarse centroids (KMeans::find_top_centroids) and keeps
//      nprobe' = max(1, min(nprobe, nlist));
//   2. for each probed list, in that order, forms the residual q - c (f32),
//      the M x ksub table lut[m][s] = metric(residual_m, codebook[m][s]) over
//      sub-vectors of ds = d / M elements, and scores every entry of the
//      list as the f32 sum of its M table values taken four at a time,
//      total += (d0 + d1) + (d2 + d3), then the remainder one by one;
//   3. keeps the k best in std's BinaryHeap compared on the heap score alone
//      (similarities negated), pushing while it holds fewer than k and
//      otherwise replacing the root (pop, then push) when the new score is
//      strictly smaller; results are popped worst first and reversed.
// Equal scores are frequent (identical codes in one list), and which of them
// survive, and in what order they come out, follows the heap's own sift
// steps, so step 3 is replayed exactly.
//
// GPU layout: the index is uploaded once (coarse centroids, codebooks, list
// offsets, ids, codes [total][M] u8, lists back to back). Step 1 runs on a
// kNN handle over the coarse centroids (vrs_ivf_find_top_centroids: stable
// (value, index) order). Steps 2-3 run in ivfpq_adc_kernel, one 128-thread
// block per query: the block builds each probed list's table in shared
// memory in the reference's pair arithmetic (vrs_exact.cuh), scores 128 list
// entries at a time (one per thread, the four-way pairing in f32 adds), and
// warp 0 replays the chunk into the heap in scan order. Once the heap is
// full only entries strictly below its root can change it, and the root
// never rises, so a ballot on the chunk-start root selects the entries lane
// 0 then applies one by one -- the same sequence of heap operations as the
// reference, at a compare per entry for the rest.
#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "vrs_exact.cuh"
#include "vrs_internal.cuh"

namespace vrs {
namespace {

constexpr int kAdcChunk = 128;                  // list entries scored per round (one per scorer)
constexpr int kAdcThreads = kAdcChunk + 32;     // four scorer warps + the replay warp
constexpr int kMaxK = 2048;           // heap capacity in shared memory
constexpr int kMaxLut = 16384;        // M * ksub table entries (64 KB)
constexpr int kMaxDim = 4096;         // residual (and its roots) in shared memory
constexpr int64_t kQueryBatch = 1 << 15;

int bad(const std::string& m) {
  set_error(VRS_ERR_INVALID_CONFIG, m);
  return VRS_ERR_INVALID_CONFIG;
}

// Device buffer owned by the index (freed with it).
struct DevArr {
  void* p = nullptr;
  size_t cap = 0;
  DevArr() = default;
  DevArr(const DevArr&) = delete;
  DevArr& operator=(const DevArr&) = delete;
  ~DevArr() {
    if (p) cudaFree(p);
  }
  int reserve(size_t bytes) {
    if (p && bytes <= cap) return VRS_OK;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    bytes = std::max<size_t>(bytes, 256);
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      p = nullptr;
      set_error(cuda_status(e), std::string("cudaMalloc: ") + cudaGetErrorString(e));
      return cuda_status(e);
    }
    cap = bytes;
    return VRS_OK;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

struct AdcArgs {
  const float* q;          // [nq][d]
  const int32_t* probe;    // [nq][P] probed list ids, best first
  int P;
  const float* coarse;     // [nlist][d]
  const float* cb;         // [M * ksub][ds]
  const float* cb_aux;     // cosine: [M * ksub] norm sums; Hellinger: [M * ksub][ds] element roots
  const float* cb_t;       // [M][ds][ksub]: the codebooks with the sub-centroid index fastest
  const int64_t* off;      // [nlist + 1]
  const uint32_t* ids;     // [total]
  const uint8_t* codes;    // [total][M]
  int d, M, ksub, ds, k;
  int nq;
  float* out_dist;         // [nq][k]
  uint32_t* out_id;        // [nq][k]
  int32_t* out_count;      // [nq]
};

// std BinaryHeap steps on three parallel shared arrays (heap score, reported
// value, id), compared on the heap score: a <= b is partial_cmp != Greater.
struct PqHeap {
  float* hs;
  float* dist;
  uint32_t* id;
  __device__ __forceinline__ static bool le(float a, float b) { return !(a > b); }
  __device__ void sift_up(int start, int pos) {
    const float eh = hs[pos], ed = dist[pos];
    const uint32_t ei = id[pos];
    while (pos > start) {
      const int parent = (pos - 1) / 2;
      if (le(eh, hs[parent])) break;
      hs[pos] = hs[parent];
      dist[pos] = dist[parent];
      id[pos] = id[parent];
      pos = parent;
    }
    hs[pos] = eh;
    dist[pos] = ed;
    id[pos] = ei;
  }
  // Towards the larger child (the right one when left <= right) down to the
  // bottom, then sift_up from there.
  __device__ void sift_down_to_bottom(int end, int pos) {
    const int start = pos;
    const float eh = hs[pos], ed = dist[pos];
    const uint32_t ei = id[pos];
    int child = 2 * pos + 1;
    while (child <= end - 2) {
      if (le(hs[child], hs[child + 1])) child += 1;
      hs[pos] = hs[child];
      dist[pos] = dist[child];
      id[pos] = id[child];
      pos = child;
      child = 2 * pos + 1;
    }
    if (child == end - 1) {
      hs[pos] = hs[child];
      dist[pos] = dist[child];
      id[pos] = id[child];
      pos = child;
    }
    hs[pos] = eh;
    dist[pos] = ed;
    id[pos] = ei;
    sift_up(start, pos);
  }
  // push at index n (the heap holds n entries before the call).
  __device__ void push(int n, float h, float dv, uint32_t iv) {
    hs[n] = h;
    dist[n] = dv;
    id[n] = iv;
    sift_up(0, n);
  }
  // pop from a heap of n >= 1 entries: the root leaves (returned), the last
  // entry takes its place and sinks.
  __device__ void pop(int n, float* h, float* dv, uint32_t* iv) {
    const int last = n - 1;
    if (last == 0) {
      *h = hs[0];
      *dv = dist[0];
      *iv = id[0];
      return;
    }
    *h = hs[0];
    *dv = dist[0];
    *iv = id[0];
    hs[0] = hs[last];
    dist[0] = dist[last];
    id[0] = id[last];
    sift_down_to_bottom(last, 0);
  }
};


// Sub-vectors shorter than 16 elements: the reference's AVX-512 kernels
// never fill a 16-lane register, their lane reductions add or take the
// maximum of zeros (+0), and only the scalar tail remains -- a sequential
// f32 sum (or maximum) from +0 with separate multiply and add, exactly as
// the general functions of vrs_exact.cuh compute it for such lengths.
// c[i * cstride] is element i of the sub-centroid (the transposed copy:
// consecutive threads read consecutive sub-centroids).
template <int METRIC>
__device__ __forceinline__ float short_key(const float* x, const float* c, int n, int cstride) {
  float r = 0.0f;
  for (int i = 0; i < n; i++) {
    const float ci = c[i * cstride];
    if (METRIC == vrs_exact::kL2 || METRIC == vrs_exact::kMaha) {
      const float d = __fsub_rn(x[i], ci);
      r = __fadd_rn(r, __fmul_rn(d, d));
    } else if (METRIC == vrs_exact::kDot) {
      r = __fadd_rn(r, __fmul_rn(x[i], ci));
    } else if (METRIC == vrs_exact::kL1) {
      r = __fadd_rn(r, fabsf(__fsub_rn(x[i], ci)));
    } else {  // kCheb
      const float d = fabsf(__fsub_rn(x[i], ci));
      if (d > r) r = d;
    }
  }
  return r;
}

// Table value lut[t], t = m * ksub + s: the reference's pair function of
// sub-vector m of the residual and sub-centroid (m, s), reported value.
template <int METRIC>
__device__ __forceinline__ float lut_value(const AdcArgs& a, const float* resid, const float* raux, int t) {
  const int m = t / a.ksub;
  const float* x = resid + m * a.ds;
  const float* c = a.cb + (size_t)t * a.ds;
  constexpr bool kShort = METRIC == vrs_exact::kL2 || METRIC == vrs_exact::kMaha || METRIC == vrs_exact::kDot ||
                          METRIC == vrs_exact::kL1 || METRIC == vrs_exact::kCheb;
  if (kShort && a.ds < 16) {
    const int sc = t - m * a.ksub;
    return vrs_exact::finish(METRIC, short_key<METRIC>(x, a.cb_t + (size_t)m * a.ds * a.ksub + sc, a.ds, a.ksub));
  }
  float key;
  if (METRIC == vrs_exact::kCos) {
    key = vrs_exact::cos_finish(vrs_exact::cos_dot(x, c, a.ds), raux[m], a.cb_aux[t]);
  } else if (METRIC == vrs_exact::kHell) {
    key = vrs_exact::hell_sum_roots(raux + m * a.ds, a.cb_aux + (size_t)t * a.ds, a.ds);
  } else {
    key = vrs_exact::rank_key(METRIC, x, c, a.ds, 0.0f, 0.0f);
  }
  return vrs_exact::finish(METRIC, key);
}

// Table build for sub-vectors of DS < 16 elements (the common PQ case): per
// sub-space m the residual slice sits in registers and thread s computes
// sub-centroids s, s + 128, ... from the transposed codebook, all DS loads
// of an entry in flight together; the arithmetic is short_key's.
template <int METRIC, int DS>
__device__ void build_table_short(const AdcArgs& a, const float* resid, float* lut, int tid) {
  for (int m = 0; m < a.M; m++) {
    float xv[DS];
#pragma unroll
    for (int e = 0; e < DS; e++) xv[e] = resid[m * DS + e];
    const float* cbm = a.cb_t + (size_t)m * DS * a.ksub;
    for (int sc = tid; sc < a.ksub; sc += kAdcChunk) {
      float cv[DS];
#pragma unroll
      for (int e = 0; e < DS; e++) cv[e] = __ldg(cbm + (size_t)e * a.ksub + sc);
      lut[m * a.ksub + sc] = vrs_exact::finish(METRIC, short_key<METRIC>(xv, cv, DS, 1));
    }
  }
}

// Builds the probed list's table into `lut` (the scorers call it).
template <int METRIC>
__device__ void build_table(const AdcArgs& a, const float* resid, const float* raux, float* lut, int tid) {
  constexpr bool kShort = METRIC == vrs_exact::kL2 || METRIC == vrs_exact::kMaha || METRIC == vrs_exact::kDot ||
                          METRIC == vrs_exact::kL1 || METRIC == vrs_exact::kCheb;
  if (kShort) {
    switch (a.ds) {
#define VRS_DS_CASE(n) \
  case n:              \
    build_table_short<METRIC, n>(a, resid, lut, tid); \
    return;
      VRS_DS_CASE(1) VRS_DS_CASE(2) VRS_DS_CASE(3) VRS_DS_CASE(4) VRS_DS_CASE(5) VRS_DS_CASE(6) VRS_DS_CASE(7)
      VRS_DS_CASE(8) VRS_DS_CASE(9) VRS_DS_CASE(10) VRS_DS_CASE(11) VRS_DS_CASE(12) VRS_DS_CASE(13)
      VRS_DS_CASE(14) VRS_DS_CASE(15)
#undef VRS_DS_CASE
      default:
        break;
    }
  }
  for (int t = tid; t < a.M * a.ksub; t += kAdcChunk) lut[t] = lut_value<METRIC>(a, resid, raux, t);
}

// Named barriers: the replay warp and the scorers hand chunk buffers to each
// other (bar.arrive on one side, bar.sync on the other, kAdcThreads threads).
// Barrier ids are immediates, so the kernel reserves only the ids it uses
// (a register id reserves all 16, which limits the blocks per SM).
template <int ID>
__device__ __forceinline__ void named_sync(int count) {
  asm volatile("bar.sync %0, %1;" ::"n"(ID), "r"(count) : "memory");
}
template <int ID>
__device__ __forceinline__ void named_arrive(int count) {
  asm volatile("bar.arrive %0, %1;" ::"n"(ID), "r"(count) : "memory");
}
constexpr int kBarFull = 1;   // + buffer: scorers -> replay warp
constexpr int kBarEmpty = 3;  // + buffer: replay warp -> scorers
constexpr int kBarTable = 5;  // scorers only: the table is built / no longer read
__device__ __forceinline__ void sync_full(int b) {
  if (b) named_sync<kBarFull + 1>(kAdcThreads); else named_sync<kBarFull>(kAdcThreads);
}
__device__ __forceinline__ void arrive_full(int b) {
  if (b) named_arrive<kBarFull + 1>(kAdcThreads); else named_arrive<kBarFull>(kAdcThreads);
}
__device__ __forceinline__ void sync_empty(int b) {
  if (b) named_sync<kBarEmpty + 1>(kAdcThreads); else named_sync<kBarEmpty>(kAdcThreads);
}
__device__ __forceinline__ void arrive_empty(int b) {
  if (b) named_arrive<kBarEmpty + 1>(kAdcThreads); else named_arrive<kBarEmpty>(kAdcThreads);
}
__device__ __forceinline__ void sync_table() { named_sync<kBarTable>(kAdcChunk); }

// One block per query. Warps 0-3 (the scorers) walk the probed lists in
// order: per list they build the table, then score 128 entries at a time
// into one of two chunk buffers. Warp 4 replays each filled buffer into the
// heap in scan order while the scorers fill the other one; both sides walk
// the same (list, chunk) sequence, so chunk j uses buffer j % 2, the
// scorers wait for the replay of chunk j - 2 before refilling it, and the
// replay of the last two chunks is never waited for (no arrive without its
// sync).
template <int METRIC>
__global__ void __launch_bounds__(kAdcThreads, 6) ivfpq_adc_kernel(AdcArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int qi = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int M = a.M, ksub = a.ksub, d = a.d, k = a.k;
  float* lut = smem;                          // [M * ksub]
  float* resid = lut + M * ksub;              // [d]
  float* raux = resid + d;                    // [d] roots (Hellinger) / [M] norm sums (cosine)
  float* c_hs = raux + d;                     // [2][128] chunk heap scores
  float* c_dist = c_hs + 2 * kAdcChunk;       // [2][128] chunk values
  uint32_t* c_id = reinterpret_cast<uint32_t*>(c_dist + 2 * kAdcChunk);  // [2][128]
  PqHeap heap;
  heap.hs = reinterpret_cast<float*>(c_id + 2 * kAdcChunk);  // [k]
  heap.dist = heap.hs + k;                                    // [k]
  heap.id = reinterpret_cast<uint32_t*>(heap.dist + k);       // [k]
  const bool hib = vrs_exact::higher_is_better(METRIC);
  const float* q = a.q + (size_t)qi * d;
  const int32_t* probe = a.probe + (size_t)qi * a.P;
  // Chunks over all probed lists (both sides need the count).
  int total = 0;
  for (int p = 0; p < a.P; p++) {
    const int c = probe[p];
    total += (int)((a.off[c + 1] - a.off[c] + kAdcChunk - 1) / kAdcChunk);
  }
  if (tid < kAdcChunk) {
    // ------------------------------------------------------------ scorers
    int chunk = 0;
    for (int p = 0; p < a.P; p++) {
      const int c = probe[p];
      const int64_t beg = a.off[c], end = a.off[c + 1];
      if (end <= beg) continue;  // empty list: skipped, as the reference does
      sync_table();  // the previous list's table is no longer read
      const float* cc = a.coarse + (size_t)c * d;
      for (int e = tid; e < d; e += kAdcChunk) {
        const float r = __fsub_rn(q[e], cc[e]);
        resid[e] = r;
        if (METRIC == vrs_exact::kHell) raux[e] = vrs_exact::root_abs(r);
      }
      sync_table();
      if (METRIC == vrs_exact::kCos) {
        for (int m = tid; m < M; m += kAdcChunk) raux[m] = vrs_exact::cos_norm_sq(resid + m * a.ds, a.ds);
        sync_table();
      }
      build_table<METRIC>(a, resid, raux, lut, tid);
      sync_table();
      for (int64_t i0 = beg; i0 < end; i0 += kAdcChunk, chunk++) {
        const int b = chunk & 1;
        if (chunk >= 2) sync_empty(b);
        const int64_t i = i0 + tid;
        if (i < end) {
          // compute_distance_with_lut: quads as (d0 + d1) + (d2 + d3), then
          // the remainder, all in f32 without contraction. With M a
          // multiple of 4 a quad's codes are one aligned 32-bit word (16
          // bytes at a time when M is a multiple of 16).
          const uint8_t* code = a.codes + (size_t)i * M;
          float total_s = 0.0f;
          int m = 0;
          auto quad = [&](uint32_t w, int mq) {
            const float d0 = lut[mq * ksub + (w & 0xff)];
            const float d1 = lut[(mq + 1) * ksub + ((w >> 8) & 0xff)];
            const float d2 = lut[(mq + 2) * ksub + ((w >> 16) & 0xff)];
            const float d3 = lut[(mq + 3) * ksub + (w >> 24)];
            total_s = __fadd_rn(total_s, __fadd_rn(__fadd_rn(d0, d1), __fadd_rn(d2, d3)));
          };
          if ((M & 15) == 0) {
            for (; m < M; m += 16) {
              const uint4 w = __ldg(reinterpret_cast<const uint4*>(code + m));
              quad(w.x, m);
              quad(w.y, m + 4);
              quad(w.z, m + 8);
              quad(w.w, m + 12);
            }
          } else if ((M & 3) == 0) {
            for (; m < M; m += 4) quad(__ldg(reinterpret_cast<const uint32_t*>(code + m)), m);
          } else {
            for (; m + 4 <= M; m += 4) {
              const float d0 = lut[m * ksub + code[m]];
              const float d1 = lut[(m + 1) * ksub + code[m + 1]];
              const float d2 = lut[(m + 2) * ksub + code[m + 2]];
              const float d3 = lut[(m + 3) * ksub + code[m + 3]];
              total_s = __fadd_rn(total_s, __fadd_rn(__fadd_rn(d0, d1), __fadd_rn(d2, d3)));
            }
            for (; m < M; m++) total_s = __fadd_rn(total_s, lut[m * ksub + code[m]]);
          }
          c_hs[b * kAdcChunk + tid] = hib ? -total_s : total_s;
          c_dist[b * kAdcChunk + tid] = total_s;
          c_id[b * kAdcChunk + tid] = a.ids[i];
        }
        arrive_full(b);
      }
    }
  } else {
    // -------------------------------------------------------- replay warp
    int n = 0;  // heap size (lane 0's view; the ballots read the root)
    int chunk = 0;
    for (int p = 0; p < a.P; p++) {
      const int c = probe[p];
      const int64_t beg = a.off[c], end = a.off[c + 1];
      for (int64_t i0 = beg; i0 < end; i0 += kAdcChunk, chunk++) {
        const int b = chunk & 1;
        const int cnt = end - i0 < kAdcChunk ? (int)(end - i0) : kAdcChunk;
        sync_full(b);
        const float* hs_b = c_hs + b * kAdcChunk;
        for (int w = 0; w < cnt; w += 32) {
          const int j = w + lane;
          const int hn = __shfl_sync(0xffffffffu, n, 0);
          // Full heap: only entries strictly below the root at the start of
          // these 32 can enter (the root never rises); filling: all of them.
          const bool cand = j < cnt && (hn < k || hs_b[j] < heap.hs[0]);
          unsigned msk = __ballot_sync(0xffffffffu, cand);
          if (lane == 0) {
            while (msk) {
              const int e = w + __ffs(msk) - 1;
              msk &= msk - 1;
              const float h = hs_b[e];
              if (n < k) {
                heap.push(n, h, c_dist[b * kAdcChunk + e], c_id[b * kAdcChunk + e]);
                n++;
              } else if (h < heap.hs[0]) {
                float th, td;
                uint32_t ti;
                heap.pop(n, &th, &td, &ti);
                heap.push(n - 1, h, c_dist[b * kAdcChunk + e], c_id[b * kAdcChunk + e]);
              }
            }
          }
          __syncwarp();
        }
        if (chunk + 2 < total) arrive_empty(b);
      }
    }
    if (lane == 0) {
      // Popped worst first; written from the back, so the row is best first.
      const int count = n;
      while (n > 0) {
        float th, td;
        uint32_t ti;
        heap.pop(n, &th, &td, &ti);
        n--;
        a.out_dist[(size_t)qi * k + n] = td;
        a.out_id[(size_t)qi * k + n] = ti;
      }
      a.out_count[qi] = count;
    }
  }
}

size_t adc_smem_bytes(int M, int ksub, int d, int k) {
  return ((size_t)M * ksub + 2 * (size_t)d + 6 * kAdcChunk + 3 * (size_t)k) * sizeof(float);
}

template <int METRIC>
int launch_adc(const AdcArgs& a, cudaStream_t s) {
  const size_t smem = adc_smem_bytes(a.M, a.ksub, a.d, a.k);
  VRS_CUDA(cudaFuncSetAttribute(ivfpq_adc_kernel<METRIC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ivfpq_adc_kernel<METRIC><<<a.nq, kAdcThreads, smem, s>>>(a);
  VRS_CUDA(cudaGetLastError());
  count_launch();
  return VRS_OK;
}

int launch_adc_metric(int metric, const AdcArgs& a, cudaStream_t s) {
  switch (metric) {
    case 0: return launch_adc<0>(a, s);
    case 1: return launch_adc<1>(a, s);
    case 2: return launch_adc<2>(a, s);
    case 3: return launch_adc<3>(a, s);
    case 4: return launch_adc<4>(a, s);
    case 5: return launch_adc<5>(a, s);
    case 6: return launch_adc<6>(a, s);
    case 7: return launch_adc<7>(a, s);
    case 8: return launch_adc<8>(a, s);
    case 9: return launch_adc<9>(a, s);
  }
  return bad("ivfpq: bad metric");
}

// Codebook side of the cosine and Hellinger tables, once per index:
// per-sub-centroid norm sums (cosine) or element roots (Hellinger).
__global__ void cb_aux_kernel(const float* __restrict__ cb, int64_t nsub, int ds, int metric, float* __restrict__ aux) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (metric == vrs_exact::kCos) {
    if (t < nsub) aux[t] = vrs_exact::cos_norm_sq(cb + t * ds, ds);
  } else if (t < nsub * ds) {
    aux[t] = vrs_exact::root_abs(cb[t]);
  }
}

}  // namespace
}  // namespace vrs

struct vrs_ivfpq {
  int64_t nlist = 0, total = 0;
  int d = 0, M = 0, ksub = 0, ds = 0, metric = 0, device = 0;
  vrs_knn* coarse_h = nullptr;  // kNN handle over the coarse centroids (probing)
  cudaStream_t stream = nullptr;
  vrs::DevArr coarse, cb, cb_aux, cb_t, off, ids, codes;
  vrs::DevArr q, probe, odist, oid, ocount;  // per search, grown on demand
  ~vrs_ivfpq() {
    if (stream) {
      cudaSetDevice(device);
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
    if (coarse_h) vrs_knn_destroy(coarse_h);
  }
};

namespace {

int upload(vrs::DevArr& dst, const void* src, size_t bytes, cudaStream_t s) {
  VRS_TRY(dst.reserve(bytes));
  if (bytes) VRS_CUDA(cudaMemcpyAsync(dst.p, src, bytes, cudaMemcpyHostToDevice, s));
  return VRS_OK;
}

}  // namespace

extern "C" int vrs_ivfpq_create(const float* coarse_centroids, int64_t nlist, int32_t d, const float* codebooks,
                                int32_t num_subvectors, int32_t sub_clusters, const int64_t* list_offsets,
                                const uint32_t* ids, const uint8_t* codes, int32_t metric, vrs_ivfpq** out) {
  using namespace vrs;
  if (!out) return bad("vrs_ivfpq_create: null out");
  *out = nullptr;
  if (d < 1 || nlist < 0 || num_subvectors < 1 || sub_clusters < 1 || metric < 0 || metric > 9)
    return bad("vrs_ivfpq_create: bad sizes or metric");
  if (d % num_subvectors != 0) return bad("vrs_ivfpq_create: dimension must be a multiple of num_subvectors");
  if (sub_clusters > 256) return bad("vrs_ivfpq_create: codes are u8, so sub_clusters <= 256");
  if ((int64_t)num_subvectors * sub_clusters > kMaxLut)
    return bad("vrs_ivfpq_create: num_subvectors * sub_clusters above " + std::to_string(kMaxLut));
  if (d > kMaxDim) return bad("vrs_ivfpq_create: dimension above " + std::to_string(kMaxDim));
  if ((nlist > 0 && (!coarse_centroids || !list_offsets)) || !codebooks)
    return bad("vrs_ivfpq_create: null buffer");
  int64_t total = 0;
  if (nlist > 0) {
    if (list_offsets[0] != 0) return bad("vrs_ivfpq_create: list_offsets[0] must be 0");
    for (int64_t c = 0; c < nlist; c++)
      if (list_offsets[c + 1] < list_offsets[c]) return bad("vrs_ivfpq_create: list_offsets must not decrease");
    total = list_offsets[nlist];
  }
  if (total > 0 && (!ids || !codes)) return bad("vrs_ivfpq_create: null ids or codes");
  for (int64_t i = 0; i < total * num_subvectors; i++)
    if (codes[i] >= sub_clusters) return bad("vrs_ivfpq_create: a code is not below sub_clusters");
  std::unique_ptr<vrs_ivfpq> h(new vrs_ivfpq());
  h->nlist = nlist;
  h->total = total;
  h->d = d;
  h->M = num_subvectors;
  h->ksub = sub_clusters;
  h->ds = d / num_subvectors;
  h->metric = metric;
  VRS_CUDA(cudaGetDevice(&h->device));
  VRS_CUDA(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  if (nlist > 0) {
    VRS_TRY(vrs_knn_create(coarse_centroids, nlist, d, 1, VRS_SHARDED, metric, &h->coarse_h));
    VRS_CUDA(cudaSetDevice(h->device));
  }
  const size_t nsub = (size_t)num_subvectors * sub_clusters;
  cudaStream_t s = h->stream;
  VRS_TRY(upload(h->coarse, coarse_centroids, (size_t)nlist * d * sizeof(float), s));
  VRS_TRY(upload(h->cb, codebooks, nsub * h->ds * sizeof(float), s));
  {
    // [M][ds][ksub] copy for coalesced table builds.
    std::vector<float> t(nsub * h->ds);
    for (int m = 0; m < num_subvectors; m++)
      for (int sc = 0; sc < sub_clusters; sc++)
        for (int e = 0; e < h->ds; e++)
          t[((size_t)m * h->ds + e) * sub_clusters + sc] = codebooks[((size_t)m * sub_clusters + sc) * h->ds + e];
    VRS_TRY(upload(h->cb_t, t.data(), t.size() * sizeof(float), s));
    VRS_CUDA(cudaStreamSynchronize(s));  // t is freed at the end of this scope
  }
  VRS_TRY(upload(h->off, list_offsets, nlist > 0 ? (size_t)(nlist + 1) * sizeof(int64_t) : 0, s));
  VRS_TRY(upload(h->ids, ids, (size_t)total * sizeof(uint32_t), s));
  VRS_TRY(upload(h->codes, codes, (size_t)total * num_subvectors, s));
  if (metric == vrs_exact::kCos || metric == vrs_exact::kHell) {
    const int64_t n_aux = metric == vrs_exact::kCos ? (int64_t)nsub : (int64_t)nsub * h->ds;
    VRS_TRY(h->cb_aux.reserve((size_t)n_aux * sizeof(float)));
    cb_aux_kernel<<<(unsigned)((n_aux + 255) / 256), 256, 0, s>>>(h->cb.as<float>(), (int64_t)nsub, h->ds, metric,
                                                                  h->cb_aux.as<float>());
    VRS_CUDA(cudaGetLastError());
    count_launch();
  }
  VRS_CUDA(cudaStreamSynchronize(s));
  *out = h.release();
  return VRS_OK;
}

extern "C" int vrs_ivfpq_search(vrs_ivfpq* h, const float* queries, int64_t nq, int32_t k, int32_t nprobe,
                                float* out_dist, uint32_t* out_id, int32_t* out_count) {
  using namespace vrs;
  if (!h) return bad("vrs_ivfpq_search: null handle");
  if (nq < 0 || k < 0 || nprobe < 0) return bad("vrs_ivfpq_search: negative nq, k or nprobe");
  if (nq == 0) return VRS_OK;
  if (!out_count) return bad("vrs_ivfpq_search: null out_count");
  // k == 0 or an empty index: every result list is empty (mod.rs:275-277).
  if (k == 0 || h->total == 0) {
    memset(out_count, 0, (size_t)nq * sizeof(int32_t));
    return VRS_OK;
  }
  if (k > kMaxK) return bad("vrs_ivfpq_search: k above " + std::to_string(kMaxK));
  if (!queries || !out_dist || !out_id) return bad("vrs_ivfpq_search: null buffer");
  // nprobe' = max(1, min(nprobe, nlist)) (mod.rs:279).
  const int32_t P = (int32_t)std::max<int64_t>(1, std::min<int64_t>(nprobe, h->nlist));
  const size_t smem = adc_smem_bytes(h->M, h->ksub, h->d, k);
  if (smem > 227 * 1024) return bad("vrs_ivfpq_search: table, residual and heap exceed shared memory");
  std::vector<float> pscore;
  std::vector<int64_t> pidx;
  std::vector<int32_t> pidx32;
  for (int64_t q0 = 0; q0 < nq; q0 += kQueryBatch) {
    const int64_t nb = std::min(kQueryBatch, nq - q0);
    // 1. Coarse probe (stable (value, index) order of find_top_centroids).
    pscore.resize((size_t)nb * P);
    pidx.resize((size_t)nb * P);
    int32_t got = 0;
    VRS_TRY(vrs_ivf_find_top_centroids(h->coarse_h, queries + q0 * h->d, nb, P, pscore.data(), pidx.data(), &got));
    if (got != P) return bad("vrs_ivfpq_search: coarse probe returned " + std::to_string(got) + " lists");
    pidx32.resize(pidx.size());
    for (size_t i = 0; i < pidx.size(); i++) pidx32[i] = (int32_t)pidx[i];
    // 2-3. Tables, scores and heaps on the GPU.
    VRS_CUDA(cudaSetDevice(h->device));
    cudaStream_t s = h->stream;
    VRS_TRY(upload(h->q, queries + q0 * h->d, (size_t)nb * h->d * sizeof(float), s));
    VRS_TRY(upload(h->probe, pidx32.data(), pidx32.size() * sizeof(int32_t), s));
    VRS_TRY(h->odist.reserve((size_t)nb * k * sizeof(float)));
    VRS_TRY(h->oid.reserve((size_t)nb * k * sizeof(uint32_t)));
    VRS_TRY(h->ocount.reserve((size_t)nb * sizeof(int32_t)));
    AdcArgs a{};
    a.q = h->q.as<float>();
    a.probe = h->probe.as<int32_t>();
    a.P = P;
    a.coarse = h->coarse.as<float>();
    a.cb = h->cb.as<float>();
    a.cb_aux = h->cb_aux.as<float>();
    a.cb_t = h->cb_t.as<float>();
    a.off = h->off.as<int64_t>();
    a.ids = h->ids.as<uint32_t>();
    a.codes = h->codes.as<uint8_t>();
    a.d = h->d;
    a.M = h->M;
    a.ksub = h->ksub;
    a.ds = h->ds;
    a.k = k;
    a.nq = (int)nb;
    a.out_dist = h->odist.as<float>();
    a.out_id = h->oid.as<uint32_t>();
    a.out_count = h->ocount.as<int32_t>();
    ProfToken t = prof_begin("ivfpq_adc", s);
    VRS_TRY(launch_adc_metric(h->metric, a, s));
    prof_end(t, s);
    VRS_CUDA(cudaMemcpyAsync(out_dist + q0 * k, a.out_dist, (size_t)nb * k * sizeof(float), cudaMemcpyDeviceToHost, s));
    VRS_CUDA(cudaMemcpyAsync(out_id + q0 * k, a.out_id, (size_t)nb * k * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    VRS_CUDA(cudaMemcpyAsync(out_count + q0, a.out_count, (size_t)nb * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    VRS_CUDA(cudaStreamSynchronize(s));
  }
  return VRS_OK;
}

extern "C" void vrs_ivfpq_destroy(vrs_ivfpq* h) { delete h; }
