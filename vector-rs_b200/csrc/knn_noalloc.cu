// knn_noalloc.cu -- exact kNN search that allocates no memory.
//
// Who needs this: callers that cannot allocate device memory at search
// time -- code running inside a captured CUDA graph region or a framework
// that forbids allocation after start-up, hosts whose device memory is
// owned by another allocator (a caching pool, a plugin host that hands out
// buffers), and hard real-time loops where cudaMalloc's latency or failure
// is not acceptable. They pass device buffers for the base, the queries and
// the results; the scan's candidate lists live in one file-scope device
// array of fixed size instead of memory allocated per call.
//
// The scratch array is kNoAllocScratchBytes (8 MiB) on every device that
// loads the library, held until the process exits. Every call uses the
// same array, so two calls that overlap on the GPU (different streams, or
// different host threads on one device) race: serialize them.
#include <mutex>

#include "vrs_exact.cuh"
#include "vrs_internal.cuh"

namespace vrs {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;

// Device-resident scratch for the per-(segment, query) candidate lists,
// their counts and the overflow flags.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[128] = {nullptr};

// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory, so the kernels get the device address looked up once per device
// (with that device current) by cudaGetSymbolAddress.
int scratch_address(void** out) {
  int dev = 0;
  VRS_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 128) {
    set_error(VRS_ERR_DEVICE_NOT_FOUND, "device ordinal out of range for the no-alloc scratch table");
    return VRS_ERR_DEVICE_NOT_FOUND;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error(cuda_status(e), std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
      return cuda_status(e);
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return VRS_OK;
}

int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace
}  // namespace vrs

extern "C" int vrs_knn_search_noalloc(const float* base, int64_t n, int32_t d, const float* queries,
                                      int64_t nq, int32_t k, int32_t metric, float* out_dist,
                                      uint32_t* out_id, int32_t* out_k, void* cuda_stream) {
  using namespace vrs;
  if (!out_k) {
    set_error(VRS_ERR_INVALID_CONFIG, "null out_k");
    return VRS_ERR_INVALID_CONFIG;
  }
  *out_k = 0;
  if (d < 1 || n < 0 || nq < 0 || k < 0 || metric < 0 || metric > 9) {
    set_error(VRS_ERR_INVALID_CONFIG, "vrs_knn_search_noalloc: bad sizes or metric");
    return VRS_ERR_INVALID_CONFIG;
  }
  if (metric == vrs_exact::kCos || metric == vrs_exact::kHell) {
    set_error(VRS_ERR_INVALID_CONFIG,
              "vrs_knn_search_noalloc: cosine and Hellinger need per-row norms/roots; use vrs_knn_search");
    return VRS_ERR_INVALID_CONFIG;
  }
  if (n > 0xfffffffeLL) {
    set_error(VRS_ERR_INVALID_CONFIG, "ids are u32: n must be < 2^32-1");
    return VRS_ERR_INVALID_CONFIG;
  }
  // No batch can hold more queries than the scratch fits at the smallest
  // list (512 candidates, one segment, one count and one flag each). Checked
  // before any size arithmetic, so the products below cannot wrap and nq
  // stays far inside int range.
  if (nq > (int64_t)((kNoAllocScratchBytes - 256) / (2 * sizeof(int) + 512 * sizeof(Cand)))) {
    set_error(VRS_ERR_INVALID_CONFIG, "vrs_knn_search_noalloc: " + std::to_string(nq) +
                                          " queries exceed the no-alloc scratch at any k; split the batch");
    return VRS_ERR_INVALID_CONFIG;
  }
  void* scratch = nullptr;
  VRS_TRY(scratch_address(&scratch));  // first call on a device: set-up
  if (nq == 0 || k == 0 || n == 0) return VRS_OK;
  if (!base || !queries || !out_dist || !out_id) {
    set_error(VRS_ERR_INVALID_CONFIG, "null buffer");
    return VRS_ERR_INVALID_CONFIG;
  }
  const int kk = (int)(k < n ? k : n);
  if (kk > 2048) {
    set_error(VRS_ERR_INVALID_CONFIG, "k' > 2048 is not supported");
    return VRS_ERR_INVALID_CONFIG;
  }
  // Same list sizing as the allocating path; as many segments as the
  // scratch holds (at most 64), at least one.
  const int cap = next_pow2(kk * 2 + 128 > 512 ? kk * 2 + 128 : 512);
  const size_t per_query_seg = (size_t)cap * sizeof(Cand) + sizeof(int);
  const size_t fixed = (size_t)nq * sizeof(int);  // overflow flags
  if (fixed + (size_t)nq * per_query_seg + 256 > kNoAllocScratchBytes) {
    const size_t max_nq = (kNoAllocScratchBytes - 256) / (per_query_seg + sizeof(int));
    set_error(VRS_ERR_INVALID_CONFIG,
              "vrs_knn_search_noalloc: " + std::to_string(nq) + " queries at k'=" + std::to_string(kk) +
                  " need more than the " + std::to_string(kNoAllocScratchBytes >> 20) +
                  " MiB no-alloc scratch (at most " + std::to_string(max_nq) +
                  " queries per call at this k); split the batch");
    return VRS_ERR_INVALID_CONFIG;
  }
  int nseg = (int)((kNoAllocScratchBytes - fixed - 256) / ((size_t)nq * per_query_seg));
  const int qtiles = (int)((nq + 31) / 32);
  const int want = (148 * 8 + qtiles - 1) / qtiles;
  if (nseg > want) nseg = want;
  if (nseg > 64) nseg = 64;
  if (nseg > 16384 / kk) nseg = 16384 / kk;
  if (nseg < 1) nseg = 1;
  int64_t seg_len = (n + nseg - 1) / nseg;
  seg_len = (seg_len + 63) / 64 * 64;
  nseg = (int)((n + seg_len - 1) / seg_len);
  // The select flags a query (and leaves its output row untouched) only
  // when its survivors exceed max_sort. The exact scan keeps at most k'
  // entries per segment and nseg <= 16384 / k' above, so nseg * k' <=
  // max_sort <= 16384 and every query's row is written; checked here,
  // before any launch, so a change to the plan cannot break it silently.
  const int ms = next_pow2(nseg * kk > 256 ? nseg * kk : 256);
  const int max_sort = ms > 16384 ? 16384 : ms;
  if (nseg * kk > max_sort) {
    set_error(VRS_ERR_DRIVER, "vrs_knn_search_noalloc: segment plan exceeds the select's sort capacity");
    return VRS_ERR_DRIVER;
  }

  unsigned char* sp = static_cast<unsigned char*>(scratch);
  int* ovf = reinterpret_cast<int*>(sp);
  int* cnt = ovf + nq;
  Cand* cand = reinterpret_cast<Cand*>(sp + (((size_t)nq + (size_t)nseg * nq) * sizeof(int) + 255) / 256 * 256);
  cudaStream_t s = (cudaStream_t)cuda_stream;
  // The array keeps the previous call's contents: counts and flags restart at zero.
  VRS_CUDA(cudaMemsetAsync(sp, 0, ((size_t)nq + (size_t)nseg * nq) * sizeof(int), s));

  KnnScanArgs a{};
  a.base = base;
  a.base_aux = nullptr;
  a.n = n;
  a.d = d;
  a.dp = d;  // caller rows are packed: row stride = d
  a.q = queries;
  a.q_aux = nullptr;
  a.q_index = nullptr;
  a.nq = (int)nq;
  a.k = kk;
  a.seg_len = seg_len;
  a.nseg = nseg;
  a.cand = cand;
  a.cnt = cnt;
  a.overflow = ovf;
  a.cap = cap;
  a.metric = metric;
  a.kind = kExactScores;
  a.rho = 1.0f;
  a.absm = nullptr;
  VRS_TRY(launch_knn_scan_exact(a, s));

  KnnSelectArgs sa{};
  sa.base = base;
  sa.base_aux = nullptr;
  sa.d = d;
  sa.dp = d;
  sa.q = queries;
  sa.q_aux = nullptr;
  sa.q_index = nullptr;
  sa.nq = (int)nq;
  sa.k = kk;
  sa.nseg = nseg;
  sa.cand = cand;
  sa.cnt = cnt;
  sa.overflow = ovf;
  sa.cap = cap;
  sa.metric = metric;
  sa.kind = kExactScores;
  sa.rho = 1.0f;
  sa.absm = nullptr;
  sa.id_offset = 0;
  sa.out_dist = out_dist;
  sa.out_id = out_id;
  sa.out_pairs = nullptr;
  sa.max_sort = max_sort;
  sa.tiny = nullptr;
  sa.n_tiny = 0;
  VRS_TRY(launch_knn_select(sa, s));
  *out_k = kk;
  return VRS_OK;
}
