// capi.cu -- the C ABI of libvrs (include/vrs.h): kNN and k-means engines,
// per-GPU shards, the single-process NCCL clique (one host thread drives
// every GPU; replaces the rayon-over-ranks loops of
// crates/vector-cuda/src/ddp/distributed_knn.rs:155-231 and
// crates/vector-cuda/src/ddp/distributed_kmeans.rs:108-330) and the
// one-process-per-GPU rank mode.
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "vrs_exact.cuh"
#include "vrs_internal.cuh"
#include "vrs_kmeans_tc.cuh"
#include "vrs_simt.cuh"
#include "vrs_tc.cuh"

namespace vrs {

static thread_local std::string g_err;

void set_error(int status, const std::string& msg) {
  (void)status;
  g_err = msg;
}

int cuda_status(cudaError_t e) {
  switch (e) {
    case cudaErrorMemoryAllocation: return VRS_ERR_OOM;
    case cudaErrorNoDevice:
    case cudaErrorInsufficientDriver: return VRS_ERR_HARDWARE_NOT_AVAILABLE;
    case cudaErrorInvalidDevice: return VRS_ERR_DEVICE_NOT_FOUND;
    default: return VRS_ERR_DRIVER;
  }
}

static int fail(int st, const std::string& m) {
  set_error(st, m);
  return st;
}

#define VRS_NCCL(call)                                                                   \
  do {                                                                                   \
    ncclResult_t _r = (call);                                                            \
    if (_r != ncclSuccess && _r != ncclInProgress)                                       \
      return ::vrs::fail(VRS_ERR_NCCL, std::string(#call) + ": " + ncclGetErrorString(_r)); \
  } while (0)

// Pinned host staging (portable across the handle's devices), grown on demand.
struct HBuf {
  void* p = nullptr;
  size_t cap = 0;
  HBuf() = default;
  HBuf(const HBuf&) = delete;
  HBuf& operator=(const HBuf&) = delete;
  ~HBuf() { release(); }
  int reserve(size_t bytes) {
    if (bytes <= cap && p) return VRS_OK;
    release();
    bytes = std::max<size_t>(bytes, 256);
    cudaError_t e = cudaHostAlloc(&p, bytes, cudaHostAllocPortable);
    if (e != cudaSuccess) {
      p = nullptr;
      return fail(cuda_status(e), "cudaHostAlloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
    cap = bytes;
    return VRS_OK;
  }
  void release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

// Growable device buffer bound to one device.
struct DBuf {
  void* p = nullptr;
  size_t cap = 0;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  ~DBuf() { release(); }
  int reserve(size_t bytes) {
    if (bytes <= cap && p) return VRS_OK;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    bytes = std::max<size_t>(bytes, 256);
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      p = nullptr;
      return fail(cuda_status(e), "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
    cap = bytes;
    return VRS_OK;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

static int round_up(int x, int m) { return (x + m - 1) / m * m; }
static int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Polls a communicator until its pending NCCL calls are enqueued (a
// non-blocking communicator may return ncclInProgress), or it reports an
// error, or `timeout_s` passes (then the communicator is aborted).
static int nccl_ready(ncclComm_t comm, double timeout_s) {
  if (!comm) return VRS_OK;
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t ar = ncclSuccess;
    ncclCommGetAsyncError(comm, &ar);
    if (ar == ncclSuccess) return VRS_OK;
    if (ar != ncclInProgress) {
      ncclCommAbort(comm);
      return fail(VRS_ERR_NCCL, std::string("NCCL async error: ") + ncclGetErrorString(ar));
    }
    const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (waited > timeout_s) {
      ncclCommAbort(comm);
      return fail(VRS_ERR_TIMEOUT, "NCCL call not enqueued within " + std::to_string(timeout_s) + " s");
    }
    // Poll (yielding the core) for the first 200 us, the usual case, then
    // every 20 us.
    if (waited > 200e-6)
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    else
      std::this_thread::yield();
  }
}

// Bounded wait for work enqueued on `s`, watching an NCCL communicator for
// asynchronous errors (a rank that died or never joined). Aborts the
// communicator and reports VRS_ERR_TIMEOUT after `timeout_s`.
static int stream_wait(cudaStream_t s, ncclComm_t comm, double timeout_s) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    if (comm) {
      ncclResult_t ar = ncclSuccess;
      ncclCommGetAsyncError(comm, &ar);
      if (ar != ncclSuccess && ar != ncclInProgress) {
        ncclCommAbort(comm);
        return fail(VRS_ERR_NCCL, std::string("NCCL async error: ") + ncclGetErrorString(ar));
      }
      if (ar == ncclSuccess) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return VRS_OK;
        if (e != cudaErrorNotReady)
          return fail(cuda_status(e), std::string("stream: ") + cudaGetErrorString(e));
      }
    } else {
      cudaError_t e = cudaStreamQuery(s);
      if (e == cudaSuccess) return VRS_OK;
      if (e != cudaErrorNotReady) return fail(cuda_status(e), std::string("stream: ") + cudaGetErrorString(e));
    }
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      if (comm) ncclCommAbort(comm);
      return fail(VRS_ERR_TIMEOUT, "device wait exceeded " + std::to_string(timeout_s) + " s");
    }
    // Poll (yielding the core) for the first millisecond, where most waits
    // end, then back off so a long wait does not occupy a core.
    if (el > 1e-3)
      std::this_thread::sleep_for(std::chrono::microseconds(comm ? 50 : 5));
    else
      std::this_thread::yield();
  }
}

static double env_timeout() {
  const char* e = getenv("VRS_TIMEOUT_S");
  return e ? atof(e) : 300.0;
}

}  // namespace vrs

using namespace vrs;

struct vrs_comm {
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0, device = 0;
  cudaStream_t stream = nullptr;
};

// ============================================================== kNN engine
namespace {

struct KnnShard {
  int device = 0;
  cudaStream_t stream = nullptr;      // stream in use
  cudaStream_t own_stream = nullptr;  // stream created for this shard
  ncclComm_t comm = nullptr;  // clique or rank communicator (not owned here)
  int64_t n_local = 0;
  int64_t offset = 0;
  DBuf base, base_aux;
  // tensor-core operands (GEMM-form metrics, d <= 128)
  bool use_tc = false;
  int num_sms = 148;
  int n_tiny = 0;
  DBuf xb, xn, xmax, tiny, ntiny;
  DBuf pb, pn;                  // pivot rows (every pivot_stride-th row)
  int64_t pivot_m = 0, pivot_stride = 1;
  DBuf tmin, ibound;            // per-search pivot-pass outputs
  DBuf ptop, ptop_all;          // smallest pivot minima per query (pool_len each): own, all shards
  float xscale = 1.0f;          // tensor-core operand scale of the base rows
  int fold_m = 0;               // exponent of the folded -|x|^2 column
  DBuf qscale;                  // per-search operand scale of each query
  DBuf qsq;                     // per-search |q|^2 from below (squared L2 / Mahalanobis)
  bool use_simt = false;        // CUDA-core scan (Manhattan, Chebyshev, Hellinger)
  // per-search scratch
  DBuf q_in, q, q_aux, cand, cnt, overflow, pairs, gathered, out_dist, out_id;
  DBuf qb, absm, err, qindex;
  DBuf mflags;                  // [c] queries of this shard's merge slice whose top-k' holds a sentinel
  DBuf all_flags;               // [G * c] every slice's flags (all-gathered)
  DBuf sl_dist, sl_id;          // [c][k'] this shard's merged slice
  DBuf q_root;                  // [nq][d] queries broadcast from rank 0 (root I/O)
  HBuf hstat;                   // pinned: [nq] flags, then the scan's error word
  int last_nq = 0, last_kk = 0, last_nseg = 0, last_cap = 0;
};

}  // namespace

struct vrs_knn {
  int64_t n_global = 0;
  int d = 0, dp = 0, metric = 0, mode = 0, g = 1;
  // Shards that split one base (row-sharded ranks or clique GPUs). With
  // parts > 1 on the tensor-core path, the shards pool their pivot minima
  // (an all-gather between the pivot pass and the main scan).
  int parts = 1;
  bool pooled_pivot = false;
  // Smallest pivot stride over the pooling shards (agreed at create time);
  // fixes the pooled bound's pivot rank, and so the all-gather's length.
  int64_t pool_stride = 1;
  std::vector<std::unique_ptr<KnnShard>> shards;
  bool rank_mode = false;
  vrs_comm* comm = nullptr;  // rank mode
  std::vector<ncclComm_t> clique;  // owned (single process, g > 1)
  ~vrs_knn() {
    for (auto& s : shards) {
      cudaSetDevice(s->device);
      cudaStreamSynchronize(s->stream);
      for (DBuf* b : {&s->base, &s->base_aux, &s->q_in, &s->q, &s->q_aux, &s->cand, &s->cnt,
                      &s->overflow, &s->pairs, &s->gathered, &s->out_dist, &s->out_id, &s->xb,
                      &s->xn, &s->xmax, &s->tiny, &s->ntiny, &s->qb, &s->absm, &s->err, &s->qindex, &s->pb,
                      &s->pn, &s->tmin, &s->ibound, &s->ptop, &s->ptop_all, &s->qscale, &s->qsq, &s->mflags,
                      &s->all_flags, &s->sl_dist, &s->sl_id, &s->q_root})
        b->release();
      s->hstat.release();
      if (s->own_stream) cudaStreamDestroy(s->own_stream);
    }
    for (ncclComm_t c : clique) ncclCommDestroy(c);
  }
};

namespace {

int valid_metric(int m) { return m >= 0 && m <= 9; }

// memcpy split over up to 8 host threads (one when the copy is small or a
// thread cannot be started): pageable or file-mapped rows reach the pinned
// staging buffer at several times one core's copy rate.
void par_memcpy(void* dst, const void* src, size_t bytes) {
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t nt = std::min<size_t>({8, hw, std::max<size_t>(1, bytes / (4u << 20))});
  if (nt <= 1) {
    memcpy(dst, src, bytes);
    return;
  }
  const size_t per = ((bytes + nt - 1) / nt + 63) & ~(size_t)63;
  std::vector<std::thread> th;
  for (size_t o = 0; o < bytes; o += per) {
    const size_t n = std::min(per, bytes - o);
    char* d = static_cast<char*>(dst) + o;
    const char* sp = static_cast<const char*>(src) + o;
    try {
      th.emplace_back([d, sp, n] { memcpy(d, sp, n); });
    } catch (...) {
      memcpy(d, sp, n);
    }
  }
  for (auto& t : th) t.join();
}

// Host rows reach the device through two pinned staging slots of 64 MB:
// while one slot's rows are copied to the device and padded (on `st`), the
// next chunk is copied from the caller's (pageable or mapped) memory into
// the other slot. A slot is refilled only after the event recorded behind
// its last device copy has completed. dst: n rows of dp floats.
// The slots (pinned host, device, events) are kept per device for the life
// of the process and reused by every upload (pinning 128 MB costs tens of
// ms, more than a whole k-means fit of 1M rows); uploads to one device take
// turns on its slots.
constexpr size_t kStageSlot = 64ull << 20;
struct StageSlots {
  std::mutex mu;
  HBuf pin[2];
  DBuf dev[2];
  cudaEvent_t ev[2] = {nullptr, nullptr};
};

StageSlots* stage_slots(int device) {
  static std::mutex g_mu;
  static StageSlots* g_slots[128] = {nullptr};  // never freed: live until exit
  if (device < 0 || device >= 128) return nullptr;
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_slots[device]) g_slots[device] = new StageSlots();
  return g_slots[device];
}

int stage_host_rows(const float* rows, int64_t n, int d, int dp, float* dst, int transform, cudaStream_t st) {
  if (n <= 0) return VRS_OK;
  int device = 0;
  VRS_CUDA(cudaGetDevice(&device));
  StageSlots* sl = stage_slots(device);
  if (!sl) return fail(VRS_ERR_DEVICE_NOT_FOUND, "device ordinal out of range for the staging slots");
  std::lock_guard<std::mutex> lk(sl->mu);
  const size_t row_bytes = (size_t)d * sizeof(float);
  const int64_t chunk = std::max<int64_t>(1, (int64_t)kStageSlot / (int64_t)row_bytes);
  const int64_t nchunks = (n + chunk - 1) / chunk;
  const size_t slot_bytes = std::max(kStageSlot, (size_t)chunk * row_bytes);
  for (int j = 0; j < 2 && j < nchunks; j++) {
    VRS_TRY(sl->pin[j].reserve(slot_bytes));
    VRS_TRY(sl->dev[j].reserve(slot_bytes));
    if (!sl->ev[j]) VRS_CUDA(cudaEventCreateWithFlags(&sl->ev[j], cudaEventDisableTiming));
  }
  int rc = VRS_OK;
  for (int64_t c = 0; c < nchunks && rc == VRS_OK; c++) {
    const int j = (int)(c & 1);
    const int64_t r0 = c * chunk, rc_rows = std::min(chunk, n - r0);
    const size_t bytes = (size_t)rc_rows * row_bytes;
    // The slot's previous copy (this upload's or an earlier one's) is done.
    if (cudaEventQuery(sl->ev[j]) != cudaSuccess) {
      cudaError_t e = cudaEventSynchronize(sl->ev[j]);
      if (e != cudaSuccess) return fail(cuda_status(e), std::string("staging: ") + cudaGetErrorString(e));
    }
    par_memcpy(sl->pin[j].p, rows + r0 * d, bytes);
    cudaError_t e = cudaMemcpyAsync(sl->dev[j].p, sl->pin[j].p, bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return fail(cuda_status(e), std::string("staging copy: ") + cudaGetErrorString(e));
    rc = launch_pad_rows(sl->dev[j].as<float>(), rc_rows, d, dp, dst + r0 * dp, transform, st);
    if (rc == VRS_OK) {
      e = cudaEventRecord(sl->ev[j], st);
      if (e != cudaSuccess) return fail(cuda_status(e), std::string("staging event: ") + cudaGetErrorString(e));
    }
  }
  // The slots are free again once `st` has run the last pad.
  cudaError_t e = cudaStreamSynchronize(st);
  if (rc == VRS_OK && e != cudaSuccess) return fail(cuda_status(e), std::string("staging: ") + cudaGetErrorString(e));
  return rc;
}

int upload_host_rows(vrs_knn* h, KnnShard* s, const float* rows, int transform) {
  return stage_host_rows(rows, s->n_local, h->d, h->dp, s->base.as<float>(), transform, s->stream);
}

// Uploads (or copies) one shard's rows into the padded layout.
int shard_upload(vrs_knn* h, KnnShard* s, const float* rows, int mem) {
  VRS_CUDA(cudaSetDevice(s->device));
  size_t nb = (size_t)std::max<int64_t>(s->n_local, 1) * h->dp * sizeof(float);
  VRS_TRY(s->base.reserve(nb));
  VRS_TRY(s->base_aux.reserve((size_t)std::max<int64_t>(s->n_local, 1) * sizeof(float)));
  if (s->n_local == 0) return VRS_OK;
  const int transform = h->metric == vrs_exact::kHell ? 1 : 0;
  if (mem == VRS_MEM_HOST) {
    VRS_TRY(upload_host_rows(h, s, rows, transform));
  } else {
    // Device rows: padded in chunks that bound each launch.
    const int64_t chunk = std::max<int64_t>(1, (int64_t)(256ll << 20) / (h->d * (int64_t)sizeof(float)));
    for (int64_t r0 = 0; r0 < s->n_local; r0 += chunk) {
      const int64_t rows_c = std::min(chunk, s->n_local - r0);
      VRS_TRY(launch_pad_rows(rows + r0 * h->d, rows_c, h->d, h->dp, s->base.as<float>() + r0 * h->dp,
                              transform, s->stream));
      VRS_CUDA(cudaStreamSynchronize(s->stream));
    }
  }
  if (h->metric == vrs_exact::kCos)
    VRS_TRY(launch_cos_norms(s->base.as<float>(), s->n_local, h->d, h->dp, s->base_aux.as<float>(),
                             s->stream));
  VRS_CUDA(cudaStreamSynchronize(s->stream));
  VRS_CUDA(cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, s->device));
  if (simt::simt_supported(h->metric, h->dp) && !getenv("VRS_DISABLE_SIMT")) s->use_simt = true;
  if (tc::tc_supported(h->metric, h->d) && !getenv("VRS_DISABLE_TC")) {
    const int d16 = tc::tc_d16(h->metric, h->d);
    const int64_t npad = (s->n_local + 127) / 128 * 128 + 128;
    VRS_TRY(s->xb.reserve((size_t)s->n_local * d16 * 2));
    VRS_TRY(s->xn.reserve((size_t)npad * sizeof(float)));
    VRS_TRY(s->xmax.reserve(sizeof(unsigned int)));
    VRS_TRY(s->tiny.reserve((size_t)tc::kTinyCap * sizeof(uint32_t)));
    VRS_TRY(s->ntiny.reserve(sizeof(int)));
    VRS_CUDA(cudaMemsetAsync(s->xn.p, 0, (size_t)npad * sizeof(float), s->stream));
    VRS_CUDA(cudaMemsetAsync(s->xmax.p, 0, sizeof(unsigned int), s->stream));
    VRS_CUDA(cudaMemsetAsync(s->ntiny.p, 0, sizeof(int), s->stream));
    // Operand scale from the largest |element| of the shard.
    {
      DBuf mx;
      VRS_TRY(mx.reserve(sizeof(float)));
      VRS_CUDA(cudaMemsetAsync(mx.p, 0, sizeof(float), s->stream));
      VRS_TRY(launch_abs_max(s->base.as<float>(), s->n_local, h->d, h->dp, mx.as<float>(), s->stream));
      float maxabs = 0.0f;
      VRS_CUDA(cudaMemcpyAsync(&maxabs, mx.p, sizeof(float), cudaMemcpyDeviceToHost, s->stream));
      VRS_CUDA(cudaStreamSynchronize(s->stream));
      s->xscale = tc::tc_base_scale(h->metric, maxabs);
      s->fold_m = tc::tc_fold_exponent(h->d, s->xscale, maxabs);
    }
    VRS_TRY(tc::tc_base_prep(s->base.as<float>(), s->n_local, h->d, h->dp, h->metric, s->xscale, s->fold_m,
                             s->xb.p, s->xn.as<float>(), s->xmax.as<unsigned int>(), s->tiny.as<uint32_t>(),
                             s->ntiny.as<int>(), tc::kTinyCap, s->stream));
    VRS_CUDA(cudaMemcpyAsync(&s->n_tiny, s->ntiny.p, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
    VRS_CUDA(cudaStreamSynchronize(s->stream));
    s->use_tc = s->n_tiny <= tc::kTinyCap;
    if (!s->use_tc) {
      s->xb.release();
    } else {
      s->pivot_m = tc::tc_pivot_rows(s->n_local, h->parts, &s->pivot_stride);
      if (s->pivot_stride > 1) {
        const int64_t ppad = (s->pivot_m + 127) / 128 * 128 + 128;
        VRS_TRY(s->pb.reserve((size_t)s->pivot_m * d16 * 2));
        VRS_TRY(s->pn.reserve((size_t)ppad * sizeof(float)));
        VRS_CUDA(cudaMemsetAsync(s->pn.p, 0, (size_t)ppad * sizeof(float), s->stream));
        VRS_TRY(tc::tc_pivot_gather(s->xb.p, s->xn.as<float>(), s->pivot_m, s->pivot_stride, d16, s->pb.p,
                                    s->pn.as<float>(), s->stream));
        VRS_CUDA(cudaStreamSynchronize(s->stream));
      }
    }
  }
  return VRS_OK;
}

struct ScanPlan {
  int nseg, cap, max_sort;
  int64_t seg_len;
};

ScanPlan plan_scan(int64_t n_local, int nq, int kk) {
  ScanPlan p;
  p.cap = next_pow2(std::max(512, 2 * kk + 128));
  int qtiles = (nq + 31) / 32;
  int want = std::max(1, (148 * 8 + qtiles - 1) / qtiles);
  int max_seg = std::max(1, std::min(64, 16384 / std::max(kk, 1)));
  int nseg = std::min(want, max_seg);
  int64_t seg_len = (n_local + nseg - 1) / nseg;
  seg_len = std::max<int64_t>(256, (seg_len + 63) / 64 * 64);
  p.nseg = (int)std::max<int64_t>(1, (n_local + seg_len - 1) / seg_len);
  p.seg_len = seg_len;
  p.max_sort = std::min(16384, next_pow2(std::max(256, p.nseg * kk)));
  return p;
}

// Local top-k' of queries already in s->q_in ([nq][d], device) against this
// shard. Writes either final results (out_dist/out_id, device) or merge pairs
// (out_pairs, device). Sets *overflow when a query needs the fallback.
// Launches the exact-order CUDA-core scan + select for `nq` query slots.
// q_index (device, nullable) maps slots to query rows of s->q; results land
// in the rows the slots name. `ovf` receives per-slot overflow flags.
// `fallback` files the launches under the knn_fallback profiling token.
int launch_exact_search(vrs_knn* h, KnnShard* s, int nq, int kk, const int* q_index, int* ovf,
                        float* out_dist, uint32_t* out_id, Cand* out_pairs, bool fallback = false) {
  cudaStream_t st = s->stream;
  ScanPlan p = plan_scan(s->n_local, nq, kk);
  VRS_TRY(s->cand.reserve((size_t)p.nseg * nq * p.cap * sizeof(Cand)));
  VRS_TRY(s->cnt.reserve((size_t)p.nseg * nq * sizeof(int)));
  VRS_CUDA(cudaMemsetAsync(s->cnt.p, 0, (size_t)p.nseg * nq * sizeof(int), st));
  KnnScanArgs a{};
  a.base = s->base.as<float>();
  a.base_aux = s->base_aux.as<float>();
  a.n = s->n_local;
  a.d = h->d;
  a.dp = h->dp;
  a.q = s->q.as<float>();
  a.q_aux = s->q_aux.as<float>();
  a.q_index = q_index;
  a.nq = nq;
  a.k = kk;
  a.seg_len = p.seg_len;
  a.nseg = p.nseg;
  a.cand = s->cand.as<Cand>();
  a.cnt = s->cnt.as<int>();
  a.overflow = ovf;
  a.cap = p.cap;
  a.metric = h->metric;
  a.kind = kExactScores;
  a.rho = 1.0f;
  a.absm = nullptr;
  if (s->n_local > 0) {
    ProfToken t = prof_begin(fallback ? "knn_fallback" : "knn_scan", st);
    VRS_TRY(launch_knn_scan_exact(a, st));
    prof_end(t, st);
  }
  KnnSelectArgs sa{};
  sa.base = a.base;
  sa.base_aux = a.base_aux;
  sa.d = h->d;
  sa.dp = h->dp;
  sa.q = a.q;
  sa.q_aux = a.q_aux;
  sa.q_index = q_index;
  sa.nq = nq;
  sa.k = kk;
  sa.nseg = s->n_local > 0 ? p.nseg : 0;
  sa.cand = a.cand;
  sa.cnt = a.cnt;
  sa.overflow = ovf;
  sa.cap = p.cap;
  sa.metric = h->metric;
  sa.kind = kExactScores;
  sa.rho = 1.0f;
  sa.absm = nullptr;
  sa.id_offset = (uint32_t)s->offset;
  sa.out_dist = out_dist;
  sa.out_id = out_id;
  sa.out_pairs = out_pairs;
  sa.max_sort = p.max_sort;
  sa.tiny = nullptr;
  sa.n_tiny = 0;
  ProfToken t = prof_begin(fallback ? "knn_fallback" : "knn_select", st);
  VRS_TRY(launch_knn_select(sa, st));
  prof_end(t, st);
  return VRS_OK;
}

// Search phases. kPhaseAll runs everything on this shard. With pooled pivot
// minima the search splits at the all-gather: kPhasePivot (query prep, pivot
// pass, this shard's k smallest minima into ptop) and kPhaseMain (bound from
// the gathered minima, main scan, select).
enum { kPhaseAll = 0, kPhasePivot = 1, kPhaseMain = 2 };

// Pivot rank of the starting bound (tc_optimistic_rank): from this shard's
// own pivot stride for a search on its own, from the agreed pool stride for
// pooled minima (the same on every shard: it is also the all-gather length).
int pool_len(const vrs_knn* h, const KnnShard* s, int kk, int phase) {
  return tc::tc_optimistic_rank(kk, phase == kPhaseAll ? s->pivot_stride : h->pool_stride);
}

// Launches the tensor-core scan + exact re-rank select for all nq queries.
int launch_tc_search(vrs_knn* h, KnnShard* s, int nq, int kk, float* out_dist, uint32_t* out_id,
                     Cand* out_pairs, int phase) {
  cudaStream_t st = s->stream;
  const int d16 = tc::tc_d16(h->metric, h->d);
  const int nq_alloc = (nq + 255) / 256 * 256;
  // The candidate pass runs on CTA pairs (cta_group::2, four lists per
  // segment); VRS_SCAN_1SM=1 selects the one-SM kernel (two lists).
  const bool pair_scan = !getenv("VRS_SCAN_1SM");
  tc::TcPlan p = pair_scan ? tc::tc_plan2(s->n_local, nq, kk, s->num_sms) : tc::tc_plan(s->n_local, nq, kk, s->num_sms);
  const int nlists = (pair_scan ? 4 : 2) * p.nseg;
  // The starting bound comes from a pivot rank below k (tc_optimistic_rank)
  // and is checked by the select: a single shard's failures are flagged for
  // the exact re-search; merge pairs carry a sentinel instead and the merge
  // decides (a pooled bound is global, so no shard can check it alone).
  const int tau_rank = pool_len(h, s, kk, phase);
  // The scan's squared-L2 scores leave |q|^2 out (see KnnSelectArgs::q_sq).
  const bool l2_scores = h->metric == vrs_exact::kL2 || h->metric == vrs_exact::kMaha;
  if (phase == kPhaseMain) goto main_phase;
  VRS_TRY(s->qb.reserve((size_t)nq_alloc * d16 * 2));
  VRS_TRY(s->absm.reserve((size_t)nq * sizeof(float)));
  VRS_TRY(s->err.reserve(sizeof(int)));
  if (nq_alloc > nq)
    VRS_CUDA(cudaMemsetAsync((char*)s->qb.p + (size_t)nq * d16 * 2, 0, (size_t)(nq_alloc - nq) * d16 * 2, st));
  VRS_CUDA(cudaMemsetAsync(s->err.p, 0, sizeof(int), st));
  VRS_TRY(s->qscale.reserve((size_t)nq * sizeof(float)));
  if (l2_scores) VRS_TRY(s->qsq.reserve((size_t)nq * sizeof(float)));
  {
    ProfToken t = prof_begin("knn_prep", st);
    VRS_TRY(tc::tc_query_prep(s->q_in.as<float>(), nq, h->d, h->dp, h->metric, s->xmax.as<unsigned int>(),
                              s->xscale, s->fold_m, s->q.as<float>(),
                              h->metric == vrs_exact::kCos ? s->q_aux.as<float>() : nullptr, s->qb.p,
                              s->qscale.as<float>(), s->absm.as<float>(), s->overflow.as<int>(),
                              l2_scores ? s->qsq.as<float>() : nullptr, st));
    prof_end(t, st);
  }
  VRS_TRY(s->ibound.reserve((size_t)nq * sizeof(float)));
  if (phase == kPhasePivot) VRS_TRY(s->ptop.reserve((size_t)nq * tau_rank * sizeof(float)));
  if (s->n_local > 0) {
    // Pivot pass: minima per column half of each tile group over every
    // pivot_stride-th row.
    const void* pb = s->pivot_stride > 1 ? s->pb.p : s->xb.p;
    const float* pn = s->pivot_stride > 1 ? s->pn.as<float>() : s->xn.as<float>();
    // On CTA pairs like the candidate pass (256-row tiles, four quarters),
    // or the one-SM kernel (128-row tiles, two halves); 256 rows per value
    // either way.
    const int ntile = (int)(pair_scan ? tc::tc_pivot_values2(s->pivot_m) : 2 * tc::tc_pivot_groups(s->pivot_m));
    VRS_TRY(s->tmin.reserve((size_t)ntile * nq * sizeof(float)));
    ProfToken t0 = prof_begin("knn_pivot", st);
    if (pair_scan) {
      tc::TcPlan pp = tc::tc_plan2(s->pivot_m, nq, kk, s->num_sms, tc::kPivotGroup);
      VRS_TRY(tc::tc_scan2(s->qb.p, nq_alloc, pb, s->pivot_m, h->d, pn, h->metric, nq, kk, pp, nullptr, nullptr,
                           s->overflow.as<int>(), s->absm.as<float>(), s->err.as<int>(), s->tmin.as<float>(),
                           nullptr, s->qscale.as<float>(), s->xscale, st));
    } else {
      tc::TcPlan pp = tc::tc_plan(s->pivot_m, nq, kk, s->num_sms, tc::kPivotGroup);
      VRS_TRY(tc::tc_scan(s->qb.p, nq_alloc, pb, s->pivot_m, h->d, pn, h->metric, nq, kk, pp, nullptr,
                          nullptr, s->overflow.as<int>(), s->absm.as<float>(), s->err.as<int>(),
                          s->tmin.as<float>(), nullptr, s->qscale.as<float>(), s->xscale, st));
    }
    if (phase == kPhasePivot)
      VRS_TRY(tc::tc_pivot_topk(s->tmin.as<float>(), ntile, nq, tau_rank, s->ptop.as<float>(), st));
    else
      VRS_TRY(tc::tc_tau(s->tmin.as<float>(), 1, 0, ntile, nq, tau_rank, s->absm.as<float>(),
                         s->ibound.as<float>(), st));
    prof_end(t0, st);
  } else if (phase == kPhasePivot) {
    VRS_CUDA(cudaMemsetAsync(s->ptop.p, 0x7f, (size_t)nq * tau_rank * sizeof(float), st));  // ~3.4e38
  }
  if (phase == kPhasePivot) return VRS_OK;
main_phase:
  if (phase == kPhaseMain && s->n_local > 0) {
    // Bound from every shard's smallest pivot minima (ptop_all, gathered).
    const int parts = h->rank_mode ? h->comm->nranks : h->g;
    ProfToken t0 = prof_begin("knn_pivot", st);
    VRS_TRY(tc::tc_tau(s->ptop_all.as<float>(), parts, (int64_t)nq * tau_rank, tau_rank, nq, tau_rank, s->absm.as<float>(),
                       s->ibound.as<float>(), st));
    prof_end(t0, st);
  }
  VRS_TRY(s->cand.reserve((size_t)nlists * nq * p.cap * sizeof(Cand)));
  VRS_TRY(s->cnt.reserve((size_t)nlists * nq * sizeof(int)));
  VRS_CUDA(cudaMemsetAsync(s->cnt.p, 0, (size_t)nlists * nq * sizeof(int), st));
  if (s->n_local > 0) {
    ProfToken t = prof_begin("knn_scan", st);
    if (pair_scan)
      VRS_TRY(tc::tc_scan2(s->qb.p, nq_alloc, s->xb.p, s->n_local, h->d, s->xn.as<float>(), h->metric, nq, kk, p,
                           s->cand.as<Cand>(), s->cnt.as<int>(), s->overflow.as<int>(), s->absm.as<float>(),
                           s->err.as<int>(), nullptr, s->ibound.as<float>(), s->qscale.as<float>(), s->xscale, st));
    else
      VRS_TRY(tc::tc_scan(s->qb.p, nq_alloc, s->xb.p, s->n_local, h->d, s->xn.as<float>(), h->metric, nq, kk,
                          p, s->cand.as<Cand>(), s->cnt.as<int>(), s->overflow.as<int>(),
                          s->absm.as<float>(), s->err.as<int>(), nullptr, s->ibound.as<float>(),
                          s->qscale.as<float>(), s->xscale, st));
    prof_end(t, st);
  }
  KnnSelectArgs sa{};
  sa.base = s->base.as<float>();
  sa.base_aux = s->base_aux.as<float>();
  sa.d = h->d;
  sa.dp = h->dp;
  sa.q = s->q.as<float>();
  sa.q_aux = s->q_aux.as<float>();
  sa.q_index = nullptr;
  sa.nq = nq;
  sa.k = kk;
  sa.nseg = s->n_local > 0 ? nlists : 0;
  sa.cand = s->cand.as<Cand>();
  sa.cnt = s->cnt.as<int>();
  sa.overflow = s->overflow.as<int>();
  sa.cap = p.cap;
  sa.metric = h->metric;
  sa.kind = kAbsMargin;
  sa.rho = 1.0f;
  sa.absm = s->absm.as<float>();
  sa.id_offset = (uint32_t)s->offset;
  sa.out_dist = out_dist;
  sa.out_id = out_id;
  sa.out_pairs = out_pairs;
  sa.max_sort = std::min(16384, next_pow2(std::max(512, nlists * (kk + 160) + s->n_tiny)));
  sa.tiny = s->tiny.as<uint32_t>();
  sa.n_tiny = h->metric == vrs_exact::kCos ? s->n_tiny : 0;
  sa.init_bound = tau_rank < kk ? s->ibound.as<float>() : nullptr;
  sa.certify = out_pairs != nullptr;
  sa.q_sq = l2_scores ? s->qsq.as<float>() : nullptr;
  ProfToken t = prof_begin("knn_select", st);
  if (nlists <= 32 && kk <= 256 && sa.n_tiny <= 256) {
    VRS_TRY(launch_knn_select_warp(sa, st));
    // Queries with more survivors than a warp holds: block select.
    sa.retry = 1;
    VRS_TRY(launch_knn_select(sa, st));
  } else {
    VRS_TRY(launch_knn_select(sa, st));
  }
  prof_end(t, st);
  return VRS_OK;
}

// CUDA-core scan (Manhattan, Chebyshev, Hellinger): pivot pass for the
// starting bounds, main scan, then the block select's exact re-rank.
int launch_simt_search(vrs_knn* h, KnnShard* s, int nq, int kk, float* out_dist, uint32_t* out_id,
                       Cand* out_pairs) {
  cudaStream_t st = s->stream;
  const float rho = simt::simt_rho(h->metric, h->d);
  simt::SimtPlan p = simt::simt_plan(s->n_local, nq, s->num_sms);
  const int cap = next_pow2(std::max(256, 2 * kk + 64));
  VRS_TRY(s->ibound.reserve((size_t)nq * sizeof(float)));
  VRS_TRY(s->cand.reserve((size_t)p.nseg * nq * cap * sizeof(Cand)));
  VRS_TRY(s->cnt.reserve((size_t)p.nseg * nq * sizeof(int)));
  VRS_CUDA(cudaMemsetAsync(s->cnt.p, 0, (size_t)p.nseg * nq * sizeof(int), st));
  if (s->n_local > 0) {
    // Pivot pass over every pstride-th row, read in place.
    int64_t pstride = 1;
    const int64_t pm = simt::simt_pivot_rows(s->n_local, kk, 1, &pstride);
    const int64_t tr = simt::simt_tile_rows();
    const int ntile = (int)((pm + tr - 1) / tr);
    simt::SimtPlan pp = simt::simt_plan(pm, nq, s->num_sms);
    VRS_TRY(s->tmin.reserve((size_t)ntile * nq * sizeof(float)));
    ProfToken t0 = prof_begin("knn_pivot", st);
    VRS_TRY(simt::simt_scan(s->base.as<float>(), pm, pstride, h->dp, s->q.as<float>(), nq, h->metric, pp, nullptr,
                            nullptr, nullptr, 0, nullptr, s->tmin.as<float>(), ntile, st));
    VRS_TRY(simt::simt_tau(s->tmin.as<float>(), ntile, nq, kk, rho, s->ibound.as<float>(), st));
    prof_end(t0, st);
    ProfToken t = prof_begin("knn_scan", st);
    VRS_TRY(simt::simt_scan(s->base.as<float>(), s->n_local, 1, h->dp, s->q.as<float>(), nq, h->metric, p,
                            s->cand.as<Cand>(), s->cnt.as<int>(), s->overflow.as<int>(), cap,
                            s->ibound.as<float>(), nullptr, 0, st));
    prof_end(t, st);
  }
  KnnSelectArgs sa{};
  sa.base = s->base.as<float>();
  sa.base_aux = s->base_aux.as<float>();
  sa.d = h->d;
  sa.dp = h->dp;
  sa.q = s->q.as<float>();
  sa.q_aux = s->q_aux.as<float>();
  sa.q_index = nullptr;
  sa.nq = nq;
  sa.k = kk;
  sa.nseg = s->n_local > 0 ? p.nseg : 0;
  sa.cand = s->cand.as<Cand>();
  sa.cnt = s->cnt.as<int>();
  sa.overflow = s->overflow.as<int>();
  sa.cap = cap;
  sa.metric = h->metric;
  sa.kind = kRelMargin;
  sa.rho = rho;
  sa.absm = nullptr;
  sa.id_offset = (uint32_t)s->offset;
  sa.out_dist = out_dist;
  sa.out_id = out_id;
  sa.out_pairs = out_pairs;
  sa.max_sort = std::min(16384, next_pow2(std::max(1024, 8 * kk + 256)));
  sa.tiny = nullptr;
  sa.n_tiny = 0;
  ProfToken t = prof_begin("knn_select", st);
  VRS_TRY(launch_knn_select(sa, st));
  prof_end(t, st);
  return VRS_OK;
}

// Phase 1 (asynchronous): local top-k' of the queries in s->q_in ([nq][d],
// device). Writes final results (out_dist/out_id) or merge pairs (out_pairs).
// `phase` splits a pooled-pivot search at its all-gather (see kPhaseAll).
int shard_search_launch(vrs_knn* h, KnnShard* s, int nq, int kk, float* out_dist, uint32_t* out_id,
                        Cand* out_pairs, int phase = kPhaseAll) {
  cudaStream_t st = s->stream;
  if (phase == kPhaseMain) {
    if (s->use_tc) return launch_tc_search(h, s, nq, kk, out_dist, out_id, out_pairs, phase);
    // A shard without rows in a pooled search: padding results only.
    return launch_exact_search(h, s, nq, kk, nullptr, s->overflow.as<int>(), out_dist, out_id, out_pairs);
  }
  VRS_TRY(s->q.reserve((size_t)nq * h->dp * sizeof(float)));
  VRS_TRY(s->q_aux.reserve((size_t)nq * sizeof(float)));
  VRS_TRY(s->overflow.reserve((size_t)(2 * nq + 1) * sizeof(int)));
  VRS_CUDA(cudaMemsetAsync(s->overflow.p, 0, (size_t)(2 * nq + 1) * sizeof(int), st));
  if (!s->use_tc) {  // the tensor-core query prep writes these itself
    ProfToken t = prof_begin("knn_prep", st);
    VRS_TRY(launch_pad_rows(s->q_in.as<float>(), nq, h->d, h->dp, s->q.as<float>(),
                            h->metric == vrs_exact::kHell ? 1 : 0, st));
    if (h->metric == vrs_exact::kCos)
      VRS_TRY(launch_cos_norms(s->q.as<float>(), nq, h->d, h->dp, s->q_aux.as<float>(), st));
    prof_end(t, st);
  }
  s->last_nq = nq;
  s->last_kk = kk;
  if (phase == kPhasePivot && !s->use_tc) {
    // A shard without rows contributes no pivot minima (~3.4e38 fillers).
    const int plen = pool_len(h, s, kk, phase);
    VRS_TRY(s->ptop.reserve((size_t)nq * plen * sizeof(float)));
    VRS_CUDA(cudaMemsetAsync(s->ptop.p, 0x7f, (size_t)nq * plen * sizeof(float), st));
    return VRS_OK;
  }
  if (s->use_tc) return launch_tc_search(h, s, nq, kk, out_dist, out_id, out_pairs, phase);
  if (s->use_simt) return launch_simt_search(h, s, nq, kk, out_dist, out_id, out_pairs);
  return launch_exact_search(h, s, nq, kk, nullptr, s->overflow.as<int>(), out_dist, out_id, out_pairs);
}

// Phase 2 (synchronous): queries whose candidate lists overflowed (or whose
// tensor-core bound does not apply) are redone with the exact-order scan.
int shard_search_finish(vrs_knn* h, KnnShard* s, float* out_dist, uint32_t* out_id, Cand* out_pairs,
                        double tmo) {
  const int nq = s->last_nq, kk = s->last_kk;
  if (nq == 0) return VRS_OK;
  std::vector<int> f(nq);
  int err = 0;
  VRS_CUDA(cudaMemcpyAsync(f.data(), s->overflow.p, (size_t)nq * sizeof(int), cudaMemcpyDeviceToHost,
                           s->stream));
  if (s->use_tc)
    VRS_CUDA(cudaMemcpyAsync(&err, s->err.p, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
  VRS_TRY(stream_wait(s->stream, nullptr, tmo));
  if (err) return fail(VRS_ERR_TIMEOUT, "tensor-core scan gave up waiting (stage code " + std::to_string(err) + ")");
  std::vector<int> idx;
  for (int i = 0; i < nq; i++)
    if (f[i]) idx.push_back(i);
  if (idx.empty()) return VRS_OK;
  const int nf = (int)idx.size();
  prof_count("knn_fallback_queries", nf);
  VRS_TRY(s->qindex.reserve((size_t)nf * sizeof(int)));
  VRS_CUDA(cudaMemcpyAsync(s->qindex.p, idx.data(), (size_t)nf * sizeof(int), cudaMemcpyHostToDevice,
                           s->stream));
  int* ovf2 = s->overflow.as<int>() + nq;
  VRS_TRY(launch_exact_search(h, s, nf, kk, s->qindex.as<int>(), ovf2, out_dist, out_id, out_pairs, true));
  std::vector<int> f2(nf);
  VRS_CUDA(cudaMemcpyAsync(f2.data(), ovf2, (size_t)nf * sizeof(int), cudaMemcpyDeviceToHost, s->stream));
  VRS_TRY(stream_wait(s->stream, nullptr, tmo));
  for (int i = 0; i < nf; i++)
    if (f2[i]) return fail(VRS_ERR_DRIVER, "exact fallback overflowed for query " + std::to_string(idx[i]));
  return VRS_OK;
}

// Pooled pivot minima need every shard with rows on the tensor-core path and
// one margin for all shards: the margins use the largest |x| of the whole
// base, since a pooled bound comes from another shard's rows. Single-process
// version: the shards' values are combined on the host.
int agree_pooled_clique(vrs_knn* h) {
  if (h->mode != VRS_SHARDED || h->g < 2 || !tc::tc_supported(h->metric, h->d) || getenv("VRS_DISABLE_TC"))
    return VRS_OK;
  unsigned int xm = 0;
  bool all = true, any = false;
  int64_t stride = INT64_MAX;
  for (auto& sp : h->shards) {
    KnnShard* s = sp.get();
    if (s->n_local == 0) continue;
    if (!s->use_tc) {
      all = false;
      continue;
    }
    any = true;
    stride = std::min(stride, s->pivot_stride);
    unsigned int v = 0;
    VRS_CUDA(cudaSetDevice(s->device));
    VRS_CUDA(cudaMemcpy(&v, s->xmax.p, sizeof(v), cudaMemcpyDeviceToHost));
    xm = std::max(xm, v);  // bits of a non-negative float order like the float
  }
  if (!all || !any) return VRS_OK;
  for (auto& sp : h->shards) {
    KnnShard* s = sp.get();
    if (!s->use_tc) continue;
    VRS_CUDA(cudaSetDevice(s->device));
    VRS_CUDA(cudaMemcpy(s->xmax.p, &xm, sizeof(xm), cudaMemcpyHostToDevice));
  }
  h->pool_stride = stride;
  h->pooled_pivot = true;
  return VRS_OK;
}

// Rank-mode version: every rank of a row-sharded handle calls this from
// vrs_knn_create_rank (a collective: an all-reduce of the TC vote and of the
// largest |x|).
int agree_pooled_rank(vrs_knn* h) {
  if (h->mode != VRS_SHARDED || h->comm->nranks < 2 || !tc::tc_supported(h->metric, h->d) ||
      getenv("VRS_DISABLE_TC"))
    return VRS_OK;
  KnnShard* s = h->shards[0].get();
  VRS_CUDA(cudaSetDevice(s->device));
  DBuf v;
  VRS_TRY(v.reserve(3 * sizeof(unsigned int)));
  // {TC vote (min), pivot stride (min; rows-less ranks are neutral), max |x| bits (max)}
  unsigned int host[3] = {(s->n_local == 0 || s->use_tc) ? 1u : 0u,
                          s->n_local > 0 ? (unsigned int)std::min<int64_t>(s->pivot_stride, 0xffffffffLL) : 0xffffffffu,
                          0u};
  if (s->use_tc) VRS_CUDA(cudaMemcpy(&host[2], s->xmax.p, sizeof(unsigned int), cudaMemcpyDeviceToHost));
  VRS_CUDA(cudaMemcpy(v.p, host, sizeof(host), cudaMemcpyHostToDevice));
  unsigned int* d = v.as<unsigned int>();
  const double tmo = env_timeout();
  VRS_NCCL(ncclGroupStart());
  VRS_NCCL(ncclAllReduce(d, d, 2, ncclUint32, ncclMin, s->comm, s->stream));
  VRS_NCCL(ncclAllReduce(d + 2, d + 2, 1, ncclUint32, ncclMax, s->comm, s->stream));
  VRS_NCCL(ncclGroupEnd());
  VRS_TRY(nccl_ready(s->comm, tmo));
  VRS_TRY(stream_wait(s->stream, s->comm, tmo));
  VRS_CUDA(cudaMemcpy(host, d, sizeof(host), cudaMemcpyDeviceToHost));
  v.release();
  if (!host[0] || !host[2]) return VRS_OK;  // a shard off the TC path, or no rows anywhere
  if (s->use_tc) VRS_CUDA(cudaMemcpy(s->xmax.p, &host[2], sizeof(unsigned int), cudaMemcpyHostToDevice));
  h->pool_stride = host[1] == 0xffffffffu ? 1 : host[1];
  h->pooled_pivot = true;
  return VRS_OK;
}

int64_t query_batch(int kk) {
  (void)kk;
  return 16384;
}

// Queries each merge participant owns: slice p is rows [p*c, (p+1)*c) of a
// batch of nb, c = ceil(nb / nranks); the pair lists are padded to
// nranks * c rows so every slice has the same size.
int slice_rows(int nb, int nranks) { return (nb + nranks - 1) / nranks; }

// Participant index of shard r: the GPU's position in a clique, the rank in
// rank mode.
int participant(const vrs_knn* h, int r) { return h->rank_mode ? h->comm->rank : r; }

// Row-sharded merge, split by query. Slots a shard flagged become sentinel
// pairs; participant p receives every shard's pairs for its own query slice
// (grouped NCCL sends and receives, its own slice by a device copy), merges
// that slice G ways in (score, id, rank) order and flags the queries whose
// top-k' holds a sentinel. The flags are all-gathered (every shard learns
// which queries to search again); the merged slices go to participant 0
// (root_only: the clique, or a rank-mode call whose results only rank 0
// reads) or to every participant. Per shard this moves 2 (G-1)/G of one
// shard's pair lists instead of receiving all G of them, and merges nb/G
// queries instead of nb.
int sharded_merge(vrs_knn* h, int nb, int kk, bool root_only, double tmo) {
  const int G = (int)h->shards.size();
  const int nranks = h->rank_mode ? h->comm->nranks : G;
  const int c = slice_rows(nb, nranks);
  const size_t sl = (size_t)c * kk;  // pairs in one slice
  std::vector<ProfToken> tg(G);
  for (int r = 0; r < G; r++) {
    KnnShard* s = h->shards[r].get();
    const int p = participant(h, r);
    VRS_CUDA(cudaSetDevice(s->device));
    VRS_TRY(launch_flag_pairs(s->overflow.as<int>(), nb, kk, s->pairs.as<Cand>(), s->stream));
    VRS_TRY(s->gathered.reserve((size_t)nranks * sl * sizeof(Cand)));
    VRS_TRY(s->sl_dist.reserve(sl * sizeof(float)));
    VRS_TRY(s->sl_id.reserve(sl * sizeof(uint32_t)));
    VRS_TRY(s->mflags.reserve((size_t)c * sizeof(int)));
    VRS_TRY(s->all_flags.reserve((size_t)nranks * c * sizeof(int)));
    VRS_TRY(s->out_dist.reserve((size_t)nranks * sl * sizeof(float)));
    VRS_TRY(s->out_id.reserve((size_t)nranks * sl * sizeof(uint32_t)));
    VRS_CUDA(cudaMemsetAsync(s->mflags.p, 0, (size_t)c * sizeof(int), s->stream));
    tg[r] = prof_begin("knn_gather", s->stream);
    VRS_CUDA(cudaMemcpyAsync(s->gathered.as<Cand>() + (size_t)p * sl, s->pairs.as<Cand>() + (size_t)p * sl,
                             sl * sizeof(Cand), cudaMemcpyDeviceToDevice, s->stream));
  }
  VRS_NCCL(ncclGroupStart());
  for (int r = 0; r < G; r++) {
    KnnShard* s = h->shards[r].get();
    const int p = participant(h, r);
    for (int j = 0; j < nranks; j++) {
      if (j == p) continue;
      VRS_NCCL(ncclSend(s->pairs.as<Cand>() + (size_t)j * sl, sl, ncclUint64, j, s->comm, s->stream));
      VRS_NCCL(ncclRecv(s->gathered.as<Cand>() + (size_t)j * sl, sl, ncclUint64, j, s->comm, s->stream));
    }
  }
  VRS_NCCL(ncclGroupEnd());
  for (int r = 0; r < G; r++) VRS_TRY(nccl_ready(h->shards[r]->comm, tmo));
  for (int r = 0; r < G; r++) {
    KnnShard* s = h->shards[r].get();
    VRS_CUDA(cudaSetDevice(s->device));
    prof_end(tg[r], s->stream);
    ProfToken t = prof_begin("knn_merge", s->stream);
    VRS_TRY(launch_merge_pairs(s->gathered.as<Cand>(), nranks, c, kk, h->metric, s->sl_dist.as<float>(),
                               s->sl_id.as<uint32_t>(), s->mflags.as<int>(), s->stream));
    prof_end(t, s->stream);
    if (root_only && participant(h, r) == 0) {
      VRS_CUDA(cudaMemcpyAsync(s->out_dist.p, s->sl_dist.p, sl * sizeof(float), cudaMemcpyDeviceToDevice,
                               s->stream));
      VRS_CUDA(cudaMemcpyAsync(s->out_id.p, s->sl_id.p, sl * sizeof(uint32_t), cudaMemcpyDeviceToDevice,
                               s->stream));
    }
  }
  VRS_NCCL(ncclGroupStart());
  for (int r = 0; r < G; r++) {
    KnnShard* s = h->shards[r].get();
    const int p = participant(h, r);
    VRS_NCCL(ncclAllGather(s->mflags.p, s->all_flags.p, (size_t)c, ncclInt32, s->comm, s->stream));
    if (!root_only) {
      VRS_NCCL(ncclAllGather(s->sl_dist.p, s->out_dist.p, sl, ncclFloat32, s->comm, s->stream));
      VRS_NCCL(ncclAllGather(s->sl_id.p, s->out_id.p, sl, ncclUint32, s->comm, s->stream));
    } else if (p != 0) {
      VRS_NCCL(ncclSend(s->sl_dist.p, sl, ncclFloat32, 0, s->comm, s->stream));
      VRS_NCCL(ncclSend(s->sl_id.p, sl, ncclUint32, 0, s->comm, s->stream));
    } else {
      for (int j = 1; j < nranks; j++) {
        VRS_NCCL(ncclRecv(s->out_dist.as<float>() + (size_t)j * sl, sl, ncclFloat32, j, s->comm, s->stream));
        VRS_NCCL(ncclRecv(s->out_id.as<uint32_t>() + (size_t)j * sl, sl, ncclUint32, j, s->comm, s->stream));
      }
    }
  }
  VRS_NCCL(ncclGroupEnd());
  for (int r = 0; r < G; r++) VRS_TRY(nccl_ready(h->shards[r]->comm, tmo));
  return VRS_OK;
}

// After every shard's search is enqueued: merge (row shards), then results,
// per-query flags and the scans' error words leave the devices behind one
// bounded wait per shard. Flagged queries (a list overflowed, a bound failed
// its check, a near-zero cosine query) are searched again with the exact
// scan on every shard and merged again; that second pass must come out
// clean. No host round trip sits between the scan and the merge. Results
// reach odst/oid from the root shard (shard 0 of a clique; rank 0 in rank
// mode with root_only) or, in rank mode without it, on every rank.
int sharded_finish(vrs_knn* h, int nb, int kk, float* odst, uint32_t* oid, cudaMemcpyKind d2h, bool root_only,
                   double tmo) {
  const int G = (int)h->shards.size();
  const int nranks = h->rank_mode ? h->comm->nranks : G;
  const bool merged = nranks > 1;
  const bool root = !h->rank_mode || !root_only || h->comm->rank == 0;
  KnnShard* s0 = h->shards[0].get();
  for (int pass = 0; pass < 2; pass++) {
    if (merged) VRS_TRY(sharded_merge(h, nb, kk, root_only || !h->rank_mode, tmo));
    for (int r = 0; r < G; r++) {
      KnnShard* s = h->shards[r].get();
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(s->hstat.reserve((size_t)(nb + 1) * sizeof(int)));
      int* hs = s->hstat.as<int>();
      hs[nb] = 0;
      if (s->use_tc && s->last_nq > 0)
        VRS_CUDA(cudaMemcpyAsync(hs + nb, s->err.p, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
      if (r == 0) {
        const int* dflags = merged ? s0->all_flags.as<int>() : s0->overflow.as<int>();
        VRS_CUDA(cudaMemcpyAsync(hs, dflags, (size_t)nb * sizeof(int), cudaMemcpyDeviceToHost, s->stream));
        if (root) {
          VRS_CUDA(cudaMemcpyAsync(odst, s0->out_dist.p, (size_t)nb * kk * sizeof(float), d2h, s->stream));
          VRS_CUDA(cudaMemcpyAsync(oid, s0->out_id.p, (size_t)nb * kk * sizeof(uint32_t), d2h, s->stream));
        }
      }
    }
    for (int r = 0; r < G; r++) {
      KnnShard* s = h->shards[r].get();
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(stream_wait(s->stream, merged ? s->comm : nullptr, tmo));
    }
    for (int r = 0; r < G; r++) {
      const int e = h->shards[r]->hstat.as<int>()[nb];
      if (e) return fail(VRS_ERR_TIMEOUT, "tensor-core scan gave up waiting (stage code " + std::to_string(e) + ")");
    }
    std::vector<int> idx;
    const int* hf = s0->hstat.as<int>();
    for (int i = 0; i < nb; i++)
      if (hf[i]) idx.push_back(i);
    if (idx.empty()) return VRS_OK;
    if (pass == 1)
      return fail(VRS_ERR_DRIVER, "exact re-search left query " + std::to_string(idx[0]) + " unresolved");
    // Exact re-search of the flagged queries on every shard; results land in
    // their rows (final results for one shard, merge pairs otherwise).
    const int nf = (int)idx.size();
    prof_count("knn_fallback_queries", nf);
    for (int r = 0; r < G; r++) {
      KnnShard* s = h->shards[r].get();
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(s->qindex.reserve((size_t)nf * sizeof(int)));
      VRS_CUDA(cudaMemcpyAsync(s->qindex.p, idx.data(), (size_t)nf * sizeof(int), cudaMemcpyHostToDevice,
                               s->stream));
      int* ovf = s->overflow.as<int>();
      VRS_CUDA(cudaMemsetAsync(ovf, 0, (size_t)(nb + nf) * sizeof(int), s->stream));
      if (!merged)
        VRS_TRY(launch_exact_search(h, s, nf, kk, s->qindex.as<int>(), ovf + nb, s->out_dist.as<float>(),
                                    s->out_id.as<uint32_t>(), nullptr, true));
      else
        VRS_TRY(launch_exact_search(h, s, nf, kk, s->qindex.as<int>(), ovf + nb, nullptr, nullptr,
                                    s->pairs.as<Cand>(), true));
      // The exact scan's own overflow flags (per flagged slot) feed the
      // second pass through the query rows they name.
      VRS_TRY(launch_scatter_flags(ovf + nb, s->qindex.as<int>(), nf, ovf, s->stream));
    }
  }
  return VRS_OK;
}

int knn_search_impl(vrs_knn* h, const float* queries, int64_t nq, int32_t k, float* out_dist,
                    uint32_t* out_id, int32_t* out_k, int mem) {
  if (!h || !out_k) return fail(VRS_ERR_INVALID_CONFIG, "null handle or out_k");
  *out_k = 0;
  if (nq < 0 || k < 0) return fail(VRS_ERR_INVALID_CONFIG, "negative nq or k");
  if (nq == 0 || k == 0 || h->n_global == 0) return VRS_OK;
  const int kk = (int)std::min<int64_t>(k, h->n_global);
  if (kk > 2048) return fail(VRS_ERR_INVALID_CONFIG, "k' > 2048 is not supported");
  const bool dev_io = (mem & VRS_MEM_DEVICE) != 0;
  // Root I/O (rank mode only): rank 0 alone holds the queries and receives
  // the results, as the one caller of the reference's search_batch does;
  // the queries reach the other ranks by an NCCL broadcast.
  const bool root_io = (mem & VRS_MEM_ROOT) != 0 && h->rank_mode && h->comm->nranks > 1;
  const bool is_root = !root_io || h->comm->rank == 0;
  if (is_root && (!queries || !out_dist || !out_id)) return fail(VRS_ERR_INVALID_CONFIG, "null buffer");
  if (dev_io && !h->rank_mode && h->shards.size() > 1)
    return fail(VRS_ERR_INVALID_CONFIG, "device buffers need a single-GPU or rank-mode handle");
  const cudaMemcpyKind h2d = dev_io ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const cudaMemcpyKind d2h = dev_io ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
  const int64_t QB = query_batch(kk);
  const double tmo = env_timeout();
  const int G = (int)h->shards.size();
  const int nranks = h->rank_mode ? h->comm->nranks : G;

  for (int64_t q0 = 0; q0 < nq; q0 += QB) {
    const int nb = (int)std::min<int64_t>(QB, nq - q0);
    const float* qsrc = is_root ? queries + q0 * h->d : nullptr;
    float* odst = is_root ? out_dist + q0 * kk : nullptr;
    uint32_t* oid = is_root ? out_id + q0 * kk : nullptr;
    cudaMemcpyKind qkind = h2d;
    if (root_io) {
      // The batch's queries from rank 0 to every rank, then read as device rows.
      KnnShard* s = h->shards[0].get();
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(s->q_root.reserve((size_t)nb * h->d * sizeof(float)));
      if (is_root)
        VRS_CUDA(cudaMemcpyAsync(s->q_root.p, qsrc, (size_t)nb * h->d * sizeof(float), h2d, s->stream));
      ProfToken tb = prof_begin("knn_gather", s->stream);
      VRS_NCCL(ncclBroadcast(s->q_root.p, s->q_root.p, (size_t)nb * h->d, ncclFloat32, 0, s->comm, s->stream));
      VRS_TRY(nccl_ready(s->comm, tmo));
      prof_end(tb, s->stream);
      qsrc = s->q_root.as<float>();
      qkind = cudaMemcpyDeviceToDevice;
    }
    if (h->mode == VRS_SHARDED) {
      // Every shard scores all queries; per-shard top-k' lists meet in an
      // all-gather and a G-way merge. With pooled pivot minima the shards
      // first exchange their k smallest pivot minima per query, so every
      // shard starts its main scan from the bound of the whole base.
      const bool pooled = h->pooled_pivot && nranks > 1;
      for (int r = 0; r < G; r++) {
        KnnShard* s = h->shards[r].get();
        VRS_CUDA(cudaSetDevice(s->device));
        VRS_TRY(s->q_in.reserve((size_t)nb * h->d * sizeof(float)));
        VRS_CUDA(cudaMemcpyAsync(s->q_in.p, qsrc, (size_t)nb * h->d * sizeof(float), qkind, s->stream));
        VRS_TRY(s->out_dist.reserve((size_t)nb * kk * sizeof(float)));
        VRS_TRY(s->out_id.reserve((size_t)nb * kk * sizeof(uint32_t)));
        if (nranks == 1) {
          VRS_TRY(shard_search_launch(h, s, nb, kk, s->out_dist.as<float>(), s->out_id.as<uint32_t>(), nullptr));
        } else {
          // Pair lists padded to whole merge slices; the padding rows hold
          // empty pairs (all bits set) whose merged rows are never read.
          const int rows = nranks * slice_rows(nb, nranks);
          VRS_TRY(s->pairs.reserve((size_t)rows * kk * sizeof(Cand)));
          if (rows > nb)
            VRS_CUDA(cudaMemsetAsync(s->pairs.as<Cand>() + (size_t)nb * kk, 0xff,
                                     (size_t)(rows - nb) * kk * sizeof(Cand), s->stream));
          VRS_TRY(shard_search_launch(h, s, nb, kk, nullptr, nullptr, s->pairs.as<Cand>(),
                                      pooled ? kPhasePivot : kPhaseAll));
        }
      }
      if (pooled) {
        const int plen = pool_len(h, h->shards[0].get(), kk, kPhasePivot);
        for (int r = 0; r < G; r++) {
          KnnShard* s = h->shards[r].get();
          VRS_CUDA(cudaSetDevice(s->device));
          VRS_TRY(s->ptop_all.reserve((size_t)nranks * nb * plen * sizeof(float)));
        }
        std::vector<ProfToken> tg(G);
        for (int r = 0; r < G; r++) {
          VRS_CUDA(cudaSetDevice(h->shards[r]->device));
          tg[r] = prof_begin("knn_gather", h->shards[r]->stream);
        }
        VRS_NCCL(ncclGroupStart());
        for (int r = 0; r < G; r++) {
          KnnShard* s = h->shards[r].get();
          VRS_NCCL(ncclAllGather(s->ptop.p, s->ptop_all.p, (size_t)nb * plen, ncclFloat32, s->comm, s->stream));
        }
        VRS_NCCL(ncclGroupEnd());
        for (int r = 0; r < G; r++) {
          VRS_CUDA(cudaSetDevice(h->shards[r]->device));
          prof_end(tg[r], h->shards[r]->stream);
        }
        for (int r = 0; r < G; r++) VRS_TRY(nccl_ready(h->shards[r]->comm, tmo));
        for (int r = 0; r < G; r++) {
          KnnShard* s = h->shards[r].get();
          VRS_CUDA(cudaSetDevice(s->device));
          VRS_TRY(shard_search_launch(h, s, nb, kk, nullptr, nullptr, s->pairs.as<Cand>(), kPhaseMain));
        }
      }
      VRS_TRY(sharded_finish(h, nb, kk, odst, oid, d2h, root_io, tmo));
    } else {
      // Replicated: query chunks of ceil(nb / ranks) (distributed_knn.rs:201-229).
      const int chunk = (nb + nranks - 1) / nranks;
      for (int r = 0; r < G; r++) {
        KnnShard* s = h->shards[r].get();
        const int rank = h->rank_mode ? h->comm->rank : r;
        const int c0 = std::min(nb, rank * chunk), c1 = std::min(nb, c0 + chunk);
        const int nc = c1 - c0;
        VRS_CUDA(cudaSetDevice(s->device));
        VRS_TRY(s->out_dist.reserve((size_t)std::max(nb, 1) * kk * sizeof(float)));
        VRS_TRY(s->out_id.reserve((size_t)std::max(nb, 1) * kk * sizeof(uint32_t)));
        VRS_TRY(s->q_in.reserve((size_t)std::max(nc, 1) * h->d * sizeof(float)));
        VRS_TRY(s->pairs.reserve((size_t)std::max(chunk, 1) * kk * sizeof(Cand)));
        if (nc > 0)
          VRS_CUDA(cudaMemcpyAsync(s->q_in.p, qsrc + (int64_t)c0 * h->d, (size_t)nc * h->d * sizeof(float),
                                   qkind, s->stream));
        s->last_nq = 0;
        if (!h->rank_mode) {
          if (nc > 0)
            VRS_TRY(shard_search_launch(h, s, nc, kk, s->out_dist.as<float>(), s->out_id.as<uint32_t>(),
                                        nullptr));
        } else {
          // Pad the chunk with empty pairs so every rank sends the same count.
          VRS_CUDA(cudaMemsetAsync(s->pairs.p, 0xff, (size_t)chunk * kk * sizeof(Cand), s->stream));
          if (nc > 0) VRS_TRY(shard_search_launch(h, s, nc, kk, nullptr, nullptr, s->pairs.as<Cand>()));
        }
      }
      for (int r = 0; r < G; r++) {
        KnnShard* s = h->shards[r].get();
        VRS_CUDA(cudaSetDevice(s->device));
        if (!h->rank_mode) {
          VRS_TRY(shard_search_finish(h, s, s->out_dist.as<float>(), s->out_id.as<uint32_t>(), nullptr, tmo));
        } else {
          VRS_TRY(shard_search_finish(h, s, nullptr, nullptr, s->pairs.as<Cand>(), tmo));
          VRS_TRY(s->gathered.reserve((size_t)nranks * chunk * kk * sizeof(Cand)));
          VRS_NCCL(ncclAllGather(s->pairs.p, s->gathered.p, (size_t)chunk * kk, ncclUint64, s->comm,
                                 s->stream));
          VRS_TRY(nccl_ready(s->comm, tmo));
          VRS_TRY(launch_finish_pairs(s->gathered.as<Cand>(), (int64_t)nb * kk, h->metric,
                                      s->out_dist.as<float>(), s->out_id.as<uint32_t>(), s->stream));
        }
      }
      for (int r = 0; r < G; r++) {
        KnnShard* s = h->shards[r].get();
        const int rank = h->rank_mode ? h->comm->rank : r;
        const int c0 = std::min(nb, rank * chunk), c1 = std::min(nb, c0 + chunk);
        VRS_CUDA(cudaSetDevice(s->device));
        VRS_TRY(stream_wait(s->stream, h->rank_mode ? s->comm : nullptr, tmo));
        if (h->rank_mode) {
          if (is_root) {
            VRS_CUDA(cudaMemcpyAsync(odst, s->out_dist.p, (size_t)nb * kk * sizeof(float), d2h, s->stream));
            VRS_CUDA(cudaMemcpyAsync(oid, s->out_id.p, (size_t)nb * kk * sizeof(uint32_t), d2h, s->stream));
          }
        } else if (c1 > c0) {
          VRS_CUDA(cudaMemcpyAsync(odst + (int64_t)c0 * kk, s->out_dist.p, (size_t)(c1 - c0) * kk * sizeof(float),
                                   d2h, s->stream));
          VRS_CUDA(cudaMemcpyAsync(oid + (int64_t)c0 * kk, s->out_id.p,
                                   (size_t)(c1 - c0) * kk * sizeof(uint32_t), d2h, s->stream));
        }
        VRS_CUDA(cudaStreamSynchronize(s->stream));
      }
    }
  }
  *out_k = kk;
  return VRS_OK;
}

int available_devices() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace

// ================================================================ C ABI
extern "C" {

int vrs_device_count(int32_t* out_count) {
  if (!out_count) return fail(VRS_ERR_INVALID_CONFIG, "null out_count");
  *out_count = available_devices();
  return VRS_OK;
}

const char* vrs_last_error(void) { return g_err.c_str(); }

int vrs_metric_higher_is_better(int32_t metric) { return vrs_exact::higher_is_better(metric) ? 1 : 0; }

int vrs_knn_create(const float* base, int64_t n, int32_t d, int32_t num_gpus, int32_t mode,
                   int32_t metric, vrs_knn** out) {
  if (!out) return fail(VRS_ERR_INVALID_CONFIG, "null out");
  *out = nullptr;
  if (num_gpus < 1) return fail(VRS_ERR_INVALID_CONFIG, "num_gpus must be at least 1");
  if (d < 1 || n < 0 || (n > 0 && !base)) return fail(VRS_ERR_INVALID_CONFIG, "bad base/dimension");
  if (n > 0xfffffffeLL) return fail(VRS_ERR_INVALID_CONFIG, "ids are u32: n must be < 2^32-1");
  if (!valid_metric(metric) || (mode != VRS_SHARDED && mode != VRS_REPLICATED))
    return fail(VRS_ERR_INVALID_CONFIG, "bad metric or mode");
  int avail = available_devices();
  if (num_gpus > avail)
    return fail(VRS_ERR_INSUFFICIENT_DEVICES, "Insufficient hardware GPUs: requested " +
                                                  std::to_string(num_gpus) + " device(s), but only " +
                                                  std::to_string(avail) + " physical GPU(s) found");
  std::unique_ptr<vrs_knn> h(new vrs_knn());
  h->n_global = n;
  h->d = d;
  h->dp = round_up(d, 8);
  h->metric = metric;
  h->mode = mode;
  const int g = (int)std::max<int64_t>(1, std::min<int64_t>(num_gpus, std::max<int64_t>(n, 1)));
  h->g = g;
  h->parts = mode == VRS_SHARDED ? g : 1;
  const int64_t chunk = (n + g - 1) / g;
  for (int r = 0; r < g; r++) {
    auto s = std::make_unique<KnnShard>();
    s->device = r;
    VRS_CUDA(cudaSetDevice(r));
    VRS_CUDA(cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking));
    s->stream = s->own_stream;
    if (mode == VRS_SHARDED) {
      int64_t b = std::min(n, r * chunk), e = std::min(n, b + chunk);
      s->offset = b;
      s->n_local = e - b;
    } else {
      s->offset = 0;
      s->n_local = n;
    }
    h->shards.push_back(std::move(s));
    VRS_TRY(shard_upload(h.get(), h->shards.back().get(), base + h->shards.back()->offset * d,
                         VRS_MEM_HOST));
  }
  if (g > 1 && mode == VRS_SHARDED) {
    h->clique.resize(g);
    std::vector<int> devs(g);
    for (int r = 0; r < g; r++) devs[r] = r;
    VRS_NCCL(ncclCommInitAll(h->clique.data(), g, devs.data()));
    for (int r = 0; r < g; r++) h->shards[r]->comm = h->clique[r];
    VRS_TRY(agree_pooled_clique(h.get()));
  }
  *out = h.release();
  return VRS_OK;
}

int vrs_knn_search(vrs_knn* h, const float* queries, int64_t nq, int32_t k, float* out_dist,
                   uint32_t* out_id, int32_t* out_k) {
  return knn_search_impl(h, queries, nq, k, out_dist, out_id, out_k, VRS_MEM_HOST);
}

int vrs_knn_search_ex(vrs_knn* h, const float* queries, int64_t nq, int32_t k, float* out_dist,
                      uint32_t* out_id, int32_t* out_k, int32_t mem) {
  if (mem & ~(VRS_MEM_DEVICE | VRS_MEM_ROOT)) return fail(VRS_ERR_INVALID_CONFIG, "bad mem flag");
  return knn_search_impl(h, queries, nq, k, out_dist, out_id, out_k, mem);
}

int vrs_knn_info(const vrs_knn* h, int64_t* num_vectors, int32_t* dimension, int32_t* num_gpus,
                 int32_t* mode, int32_t* metric) {
  if (!h) return fail(VRS_ERR_INVALID_CONFIG, "null handle");
  if (num_vectors) *num_vectors = h->n_global;
  if (dimension) *dimension = h->d;
  if (num_gpus) *num_gpus = h->rank_mode ? h->comm->nranks : h->g;
  if (mode) *mode = h->mode;
  if (metric) *metric = h->metric;
  return VRS_OK;
}

void vrs_knn_destroy(vrs_knn* h) { delete h; }

int vrs_knn_set_stream(vrs_knn* h, void* cuda_stream) {
  if (!h) return fail(VRS_ERR_INVALID_CONFIG, "null handle");
  if (h->shards.size() != 1) return fail(VRS_ERR_INVALID_CONFIG, "set_stream needs a single-GPU or rank-mode handle");
  KnnShard* s = h->shards[0].get();
  VRS_CUDA(cudaSetDevice(s->device));
  VRS_CUDA(cudaStreamSynchronize(s->stream));
  s->stream = cuda_stream ? (cudaStream_t)cuda_stream : s->own_stream;
  return VRS_OK;
}

int vrs_comm_unique_id(uint8_t out_id[128]) {
  if (!out_id) return fail(VRS_ERR_INVALID_CONFIG, "null id buffer");
  ncclUniqueId id;
  VRS_NCCL(ncclGetUniqueId(&id));
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  memcpy(out_id, &id, 128);
  return VRS_OK;
}

int vrs_comm_init(const uint8_t id[128], int32_t nranks, int32_t rank, int32_t device, vrs_comm** out) {
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(VRS_ERR_INVALID_CONFIG, "bad comm arguments");
  *out = nullptr;
  int avail = available_devices();
  if (device < 0 || device >= avail)
    return fail(VRS_ERR_DEVICE_NOT_FOUND, "CUDA device with ordinal " + std::to_string(device) +
                                              " was not found or could not be initialized");
  std::unique_ptr<vrs_comm> c(new vrs_comm());
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  VRS_CUDA(cudaSetDevice(device));
  VRS_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  ncclUniqueId uid;
  memcpy(&uid, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress)
    return fail(VRS_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclCommGetAsyncError(c->comm, &st);
    if (st == ncclSuccess) break;
    if (st != ncclInProgress) {
      ncclCommAbort(c->comm);
      return fail(VRS_ERR_NCCL, std::string("NCCL init: ") + ncclGetErrorString(st));
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > env_timeout()) {
      ncclCommAbort(c->comm);
      return fail(VRS_ERR_TIMEOUT, "NCCL init timed out (a rank never joined)");
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  *out = c.release();
  return VRS_OK;
}

void vrs_comm_destroy(vrs_comm* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->comm) ncclCommDestroy(c->comm);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

int vrs_knn_create_rank(vrs_comm* comm, const float* shard, int64_t n_local, int64_t global_offset,
                        int64_t n_global, int32_t d, int32_t mode, int32_t metric, int32_t mem,
                        vrs_knn** out) {
  if (!out || !comm) return fail(VRS_ERR_INVALID_CONFIG, "null comm or out");
  *out = nullptr;
  if (d < 1 || n_local < 0 || n_global < n_local || global_offset < 0 || (n_local > 0 && !shard))
    return fail(VRS_ERR_INVALID_CONFIG, "bad shard arguments");
  if (n_global > 0xfffffffeLL) return fail(VRS_ERR_INVALID_CONFIG, "ids are u32: n must be < 2^32-1");
  if (!valid_metric(metric) || (mode != VRS_SHARDED && mode != VRS_REPLICATED))
    return fail(VRS_ERR_INVALID_CONFIG, "bad metric or mode");
  if (mem != VRS_MEM_HOST && mem != VRS_MEM_DEVICE) return fail(VRS_ERR_INVALID_CONFIG, "bad mem flag");
  std::unique_ptr<vrs_knn> h(new vrs_knn());
  h->n_global = n_global;
  h->d = d;
  h->dp = round_up(d, 8);
  h->metric = metric;
  h->mode = mode;
  h->g = 1;
  h->rank_mode = true;
  h->comm = comm;
  h->parts = mode == VRS_SHARDED ? comm->nranks : 1;
  auto s = std::make_unique<KnnShard>();
  s->device = comm->device;
  s->comm = comm->comm;
  s->n_local = n_local;
  s->offset = global_offset;
  VRS_CUDA(cudaSetDevice(comm->device));
  VRS_CUDA(cudaStreamCreateWithFlags(&s->own_stream, cudaStreamNonBlocking));
  s->stream = s->own_stream;
  h->shards.push_back(std::move(s));
  VRS_TRY(shard_upload(h.get(), h->shards[0].get(), shard, mem));
  VRS_TRY(agree_pooled_rank(h.get()));
  *out = h.release();
  return VRS_OK;
}

}  // extern "C"

// ============================================================ k-means
namespace {

constexpr int kSumSlots = 513;  // launch_sum_f64 partials + result

struct KmShard {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  ncclComm_t comm = nullptr;
  int64_t n_local = 0;
  DBuf x, xr, x_aux, assign, dist, acc, cent, cent_r, cent_aux, shift, scal, red;
  // tensor-core assignment operands
  bool use_tc = false;
  DBuf xb, xq, xtiny, cb, cn, cmax, res, cands, err, ctiny;
  DBuf flags;  // finalize lists: [count F, count M, F indices (n), M indices (n)]
  DBuf segws;  // counting-sort workspace of the centroid sums
  HBuf hstat;  // pinned: {assignment error word, max centroid shift} per iteration
  DBuf cent_prev;        // centroids the latest assignment was made against
  DBuf pscore, ibound;   // squared L2: score bound of each point's assignment; next step's starting bound
  bool last_tc = false;  // the latest assignment took the tensor-core path
  ~KmShard() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (DBuf* b : {&x, &xr, &x_aux, &assign, &dist, &acc, &cent, &cent_r, &cent_aux, &shift, &scal, &red, &xb,
                    &xq, &xtiny, &cb, &cn, &cmax, &res, &cands, &err, &ctiny, &segws, &flags, &cent_prev, &pscore,
                    &ibound})
      b->release();
    hstat.release();
    if (stream) cudaStreamDestroy(stream);
  }
};

struct KmParams {
  int64_t n_global;
  int d, dp, k, max_iters, metric;
  float tol;
  int nranks;  // participants in the all-reduce (shards in a clique, or ranks)
  bool rank_mode;
};

int km_prepare_shard(const KmParams& P, KmShard* s, const float* rows, int mem) {
  VRS_CUDA(cudaSetDevice(s->device));
  const size_t nx = (size_t)std::max<int64_t>(s->n_local, 1);
  VRS_TRY(s->x.reserve(nx * P.dp * sizeof(float)));
  VRS_TRY(s->assign.reserve(nx * sizeof(int32_t)));
  VRS_TRY(s->dist.reserve(nx * sizeof(float)));
  VRS_TRY(s->x_aux.reserve(nx * sizeof(float)));
  VRS_TRY(s->acc.reserve(((size_t)P.k * P.dp + P.k) * sizeof(unsigned long long)));
  VRS_TRY(s->cent.reserve((size_t)P.k * P.dp * sizeof(float)));
  VRS_TRY(s->cent_r.reserve((size_t)P.k * P.dp * sizeof(float)));
  VRS_TRY(s->cent_aux.reserve((size_t)P.k * sizeof(float)));
  VRS_TRY(s->shift.reserve((size_t)P.k * sizeof(float)));
  VRS_TRY(s->scal.reserve(4 * sizeof(float)));
  VRS_TRY(s->red.reserve(kSumSlots * sizeof(double)));
  if (s->n_local > 0) {
    if (mem == VRS_MEM_HOST) {
      // Pinned staging slots with a multi-threaded host copy (as the kNN upload).
      VRS_TRY(stage_host_rows(rows, s->n_local, P.d, P.dp, s->x.as<float>(), 0, s->stream));
    } else {
      VRS_TRY(launch_pad_rows(rows, s->n_local, P.d, P.dp, s->x.as<float>(), 0, s->stream));
      VRS_CUDA(cudaStreamSynchronize(s->stream));
    }
    if (P.metric == vrs_exact::kHell) {
      VRS_TRY(s->xr.reserve(nx * P.dp * sizeof(float)));
      VRS_TRY(launch_pad_rows(s->x.as<float>(), s->n_local, P.dp, P.dp, s->xr.as<float>(), 1, s->stream));
    }
    if (P.metric == vrs_exact::kCos)
      VRS_TRY(launch_cos_norms(s->x.as<float>(), s->n_local, P.d, P.dp, s->x_aux.as<float>(), s->stream));
  }
  VRS_CUDA(cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, s->device));
  if (kmtc::supported(P.metric, P.d) && !getenv("VRS_DISABLE_TC") && s->n_local > 0) {
    const int d16 = (P.d + 15) / 16 * 16;
    const int64_t kpad = (P.k + 127) / 128 * 128 + 128;
    VRS_TRY(s->xb.reserve((size_t)s->n_local * d16 * 2));
    VRS_TRY(s->xq.reserve(nx * sizeof(float)));
    VRS_TRY(s->xtiny.reserve(nx * sizeof(int)));
    VRS_TRY(s->cb.reserve((size_t)P.k * d16 * 2));
    VRS_TRY(s->cn.reserve((size_t)kpad * sizeof(float)));
    VRS_TRY(s->cmax.reserve(2 * sizeof(unsigned int)));
    VRS_TRY(s->ctiny.reserve(sizeof(int)));
    VRS_TRY(s->res.reserve(nx * 2 * sizeof(kmtc::Res)));
    VRS_TRY(s->cands.reserve(kmtc::group_bytes(nx)));
    VRS_TRY(s->flags.reserve((2 * nx + 2) * sizeof(int)));
    VRS_TRY(s->err.reserve(sizeof(int)));
    if (P.metric == vrs_exact::kL2 || P.metric == vrs_exact::kMaha) {
      VRS_TRY(s->pscore.reserve(nx * sizeof(float)));
      VRS_TRY(s->ibound.reserve(nx * sizeof(float)));
    }
    VRS_CUDA(cudaMemsetAsync(s->cn.p, 0, (size_t)kpad * sizeof(float), s->stream));
    s->use_tc = true;  // point operands are prepared in km_run, once the global max |x| is known
  }
  return VRS_OK;
}

// Shared Lloyd loop over 1..G shards (clique) or one shard per rank.
int km_run(const KmParams& P, std::vector<KmShard*>& shards, const float* init_host,
           float* out_centroids, int32_t* out_assign_local, int32_t* out_iters, double* out_inertia) {
  const double tmo = env_timeout();
  const int G = (int)shards.size();
  const bool coll = P.nranks > 1;
  // Initial centroids (padded) on every shard.
  {
    std::vector<float> padded((size_t)P.k * P.dp, 0.0f);
    for (int c = 0; c < P.k; c++)
      memcpy(&padded[(size_t)c * P.dp], init_host + (size_t)c * P.d, P.d * sizeof(float));
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_CUDA(cudaMemcpyAsync(s->cent.p, padded.data(), padded.size() * sizeof(float),
                               cudaMemcpyHostToDevice, s->stream));
      VRS_CUDA(cudaStreamSynchronize(s->stream));
    }
  }
  // Fixed-point scale from the global max |x|.
  float gmax = 0.0f;
  for (KmShard* s : shards) {
    VRS_CUDA(cudaSetDevice(s->device));
    VRS_TRY(launch_abs_max(s->x.as<float>(), s->n_local, P.d, P.dp, s->scal.as<float>(), s->stream));
  }
  if (coll) {
    VRS_NCCL(ncclGroupStart());
    for (KmShard* s : shards)
      VRS_NCCL(ncclAllReduce(s->scal.p, s->scal.p, 1, ncclFloat32, ncclMax, s->comm, s->stream));
    VRS_NCCL(ncclGroupEnd());
  }
  for (KmShard* s : shards) {
    VRS_CUDA(cudaSetDevice(s->device));
    VRS_TRY(stream_wait(s->stream, coll ? s->comm : nullptr, tmo));
    float m = 0;
    VRS_CUDA(cudaMemcpy(&m, s->scal.p, sizeof(float), cudaMemcpyDeviceToHost));
    gmax = std::max(gmax, m);
  }
  int scale_exp = 0;
  if (gmax > 0.0f) {
    double lim = 61.0 - std::log2((double)std::max<int64_t>(P.n_global, 1) * (double)gmax);
    scale_exp = (int)std::floor(lim);
    scale_exp = std::max(-200, std::min(100, scale_exp));
  }
  // Tensor-core operands: fp16 of value * op_scale, a power of two putting
  // the largest element in [2^13, 2^14) (centroids are means of points, so
  // they fit too); cosine rows are normalised and use 1.
  // Empty clusters keep their initial centroid, so the initial centroids
  // count too.
  float omax = gmax;
  for (size_t i = 0; i < (size_t)P.k * P.d; i++) omax = std::max(omax, std::fabs(init_host[i]));
  float op_scale = 1.0f;
  if (P.metric != vrs_exact::kCos && omax > 0.0f && std::isfinite(omax))
    op_scale = std::ldexp(1.0f, std::max(-100, std::min(100, 13 - std::ilogb(omax))));
  for (KmShard* s : shards) {
    if (!s->use_tc) continue;
    VRS_CUDA(cudaSetDevice(s->device));
    VRS_TRY(kmtc::prep_rows(s->x.as<float>(), s->n_local, P.d, P.dp, P.metric, op_scale, s->xb.p, nullptr,
                            s->xq.as<float>(), nullptr, s->xtiny.as<int>(), nullptr, s->stream));
  }
  const size_t acc_elems = (size_t)P.k * P.dp + P.k;
  int iters = 0;
  // The Lloyd loop proper (upload, operand prep and initial centroids are
  // outside it), timed on shard 0's stream as profile name "kmeans_loop".
  VRS_CUDA(cudaSetDevice(shards[0]->device));
  for (KmShard* s : shards)
    if (s->use_tc) {
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(s->cent_prev.reserve((size_t)P.k * P.dp * sizeof(float)));
    }
  ProfToken tloop = prof_begin("kmeans_loop", shards[0]->stream);
  for (int it = 0; it < P.max_iters; it++) {
    iters = it + 1;
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      const float* cent_ops = s->cent.as<float>();
      const float* x_ops = s->x.as<float>();
      if (P.metric == vrs_exact::kHell) {
        VRS_TRY(launch_pad_rows(s->cent.as<float>(), P.k, P.dp, P.dp, s->cent_r.as<float>(), 1, s->stream));
        cent_ops = s->cent_r.as<float>();
        x_ops = s->xr.as<float>();
      }
      if (P.metric == vrs_exact::kCos)
        VRS_TRY(launch_cos_norms(s->cent.as<float>(), P.k, P.d, P.dp, s->cent_aux.as<float>(), s->stream));
      bool tc_done = false;
      if (s->use_tc) {
        // Centroid operands for this iteration; a near-zero cosine centroid
        // sends the iteration to the exact path.
        int any_tiny = 0;
        VRS_CUDA(cudaMemsetAsync(s->cmax.p, 0, 2 * sizeof(unsigned int), s->stream));
        VRS_CUDA(cudaMemsetAsync(s->ctiny.p, 0, sizeof(int), s->stream));
        VRS_TRY(kmtc::prep_rows(s->cent.as<float>(), P.k, P.d, P.dp, P.metric, op_scale, s->cb.p,
                                (P.metric == vrs_exact::kL2 || P.metric == vrs_exact::kMaha) ? s->cn.as<float>()
                                                                                              : nullptr,
                                nullptr, s->cmax.as<unsigned int>(), nullptr, s->ctiny.as<int>(), s->stream));
        if (P.metric == vrs_exact::kCos) {
          VRS_CUDA(cudaMemcpyAsync(&any_tiny, s->ctiny.p, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
          VRS_CUDA(cudaStreamSynchronize(s->stream));
        }
        if (!any_tiny) {
          VRS_CUDA(cudaMemsetAsync(s->err.p, 0, sizeof(int), s->stream));
          // Squared L2 after a tensor-core step: every point starts from the
          // bound its last assignment and that centroid's shift give.
          const bool l2 = P.metric == vrs_exact::kL2 || P.metric == vrs_exact::kMaha;
          const bool start = l2 && it > 0 && s->last_tc;
          ProfToken t = prof_begin("kmeans_assign", s->stream);
          if (start)
            VRS_TRY(kmtc::start_bound(s->n_local, s->assign.as<int32_t>(), s->pscore.as<float>(),
                                      s->xq.as<float>(), s->shift.as<float>(), s->ibound.as<float>(), s->stream));
          VRS_TRY(kmtc::assign(s->xb.p, s->n_local, s->cb.p, P.k, P.d, s->cn.as<float>(), s->xq.as<float>(),
                               s->cmax.as<unsigned int>(), P.metric, op_scale, s->res.as<kmtc::Res>(),
                               s->cands.p, s->err.as<int>(), s->num_sms,
                               start ? s->ibound.as<float>() : nullptr, s->stream));
          prof_end(t, s->stream);
          ProfToken t2 = prof_begin("kmeans_finalize", s->stream);
          VRS_TRY(kmtc::finalize(s->x.as<float>(), s->n_local, P.d, P.dp, s->cent.as<float>(),
                                 s->cent_aux.as<float>(), s->x_aux.as<float>(), P.k, s->xq.as<float>(),
                                 s->cmax.as<unsigned int>(), P.metric, s->res.as<kmtc::Res>(),
                                 s->cands.p,
                                 P.metric == vrs_exact::kCos ? s->xtiny.as<int>() : nullptr,
                                 s->assign.as<int32_t>(), s->dist.as<float>(), s->flags.as<int>(), s->num_sms,
                                 op_scale, l2 ? s->pscore.as<float>() : nullptr, s->stream));
          prof_end(t2, s->stream);
          tc_done = true;
        }
      }
      s->last_tc = tc_done;
      if (!tc_done) {
        ProfToken t = prof_begin("kmeans_assign", s->stream);
        VRS_TRY(launch_kmeans_assign_exact(x_ops, s->n_local, P.d, P.dp, cent_ops, s->cent_aux.as<float>(),
                                           s->x_aux.as<float>(), P.k, P.metric, s->assign.as<int32_t>(),
                                           s->dist.as<float>(), s->stream));
        prof_end(t, s->stream);
      }
      VRS_CUDA(cudaMemsetAsync(s->acc.p, 0, acc_elems * sizeof(unsigned long long), s->stream));
      unsigned long long* sums = s->acc.as<unsigned long long>();
      VRS_TRY(s->segws.reserve(kmeans_segsum_ws_bytes(s->n_local, P.k)));
      ProfToken ts = prof_begin("kmeans_sums", s->stream);
      VRS_TRY(launch_kmeans_segsum(s->x.as<float>(), s->n_local, P.d, P.dp, s->assign.as<int32_t>(), P.k,
                                   scale_exp, sums, sums + (size_t)P.k * P.dp, s->segws.as<int>(), s->stream));
      prof_end(ts, s->stream);
    }
    if (coll) {
      VRS_NCCL(ncclGroupStart());
      for (KmShard* s : shards)
        VRS_NCCL(ncclAllReduce(s->acc.p, s->acc.p, acc_elems, ncclUint64, ncclSum, s->comm, s->stream));
      VRS_NCCL(ncclGroupEnd());
      for (KmShard* s : shards) VRS_TRY(nccl_ready(s->comm, tmo));
    }
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      unsigned long long* sums = s->acc.as<unsigned long long>();
      if (s->last_tc) {
        // The tensor-core finalize leaves single-candidate points without
        // an exact distance; keep the centroids they were assigned against
        // for the inertia pass after the loop.
        VRS_CUDA(cudaMemcpyAsync(s->cent_prev.p, s->cent.p, (size_t)P.k * P.dp * sizeof(float),
                                 cudaMemcpyDeviceToDevice, s->stream));
      }
      ProfToken t = prof_begin("kmeans_update", s->stream);
      VRS_TRY(launch_kmeans_update(sums, sums + (size_t)P.k * P.dp, P.k, P.d, P.dp, scale_exp,
                                   s->cent.as<float>(), s->shift.as<float>(), s->scal.as<float>() + 1,
                                   s->stream));
      prof_end(t, s->stream);
    }
    // The error words and the convergence value ride the same bounded wait
    // (pinned copies queued behind the update), one per shard.
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(s->hstat.reserve(2 * sizeof(int)));
      int* hs = s->hstat.as<int>();
      hs[0] = 0;
      if (s->use_tc) VRS_CUDA(cudaMemcpyAsync(hs, s->err.p, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
      if (s == shards[0])
        VRS_CUDA(cudaMemcpyAsync(hs + 1, s->scal.as<float>() + 1, sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    }
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      VRS_TRY(stream_wait(s->stream, coll ? s->comm : nullptr, tmo));
    }
    for (KmShard* s : shards) {
      const int err = s->hstat.as<int>()[0];
      if (err)
        return fail(VRS_ERR_TIMEOUT, "tensor-core k-means assignment gave up waiting (stage code " +
                                         std::to_string(err) + ")");
    }
    float max_shift = 0.0f;
    std::memcpy(&max_shift, shards[0]->hstat.as<int>() + 1, sizeof(float));
    if (max_shift <= P.tol) break;
  }
  VRS_CUDA(cudaSetDevice(shards[0]->device));
  prof_end(tloop, shards[0]->stream);
  // Inertia of the last assignment step: deterministic per-shard f64 sums,
  // added in rank order.
  double inertia = 0.0;
  if (iters > 0) {
    std::vector<double> parts;
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      if (s->last_tc)
        VRS_TRY(kmtc::fill_dist(s->x.as<float>(), s->n_local, P.d, P.dp, s->cent_prev.as<float>(),
                                s->cent_aux.as<float>(), s->x_aux.as<float>(), P.metric, s->assign.as<int32_t>(),
                                s->dist.as<float>(), s->stream));
      VRS_TRY(launch_sum_f64(s->dist.as<float>(), s->n_local, s->red.as<double>(), s->stream));
    }
    if (P.rank_mode && coll) {
      KmShard* s = shards[0];
      DBuf g;
      VRS_TRY(g.reserve((size_t)P.nranks * sizeof(double)));
      VRS_NCCL(ncclAllGather(s->red.as<double>() + (kSumSlots - 1), g.p, 1, ncclFloat64, s->comm, s->stream));
      VRS_TRY(stream_wait(s->stream, s->comm, tmo));
      parts.resize(P.nranks);
      VRS_CUDA(cudaMemcpy(parts.data(), g.p, P.nranks * sizeof(double), cudaMemcpyDeviceToHost));
      g.release();
    } else {
      for (KmShard* s : shards) {
        VRS_CUDA(cudaSetDevice(s->device));
        VRS_TRY(stream_wait(s->stream, nullptr, tmo));
        double v = 0;
        VRS_CUDA(cudaMemcpy(&v, s->red.as<double>() + (kSumSlots - 1), sizeof(double), cudaMemcpyDeviceToHost));
        parts.push_back(v);
      }
    }
    for (double v : parts) inertia += v;
  }
  // Outputs.
  {
    KmShard* s0 = shards[0];
    VRS_CUDA(cudaSetDevice(s0->device));
    std::vector<float> padded((size_t)P.k * P.dp);
    VRS_CUDA(cudaMemcpy(padded.data(), s0->cent.p, padded.size() * sizeof(float), cudaMemcpyDeviceToHost));
    for (int c = 0; c < P.k; c++)
      memcpy(out_centroids + (size_t)c * P.d, &padded[(size_t)c * P.dp], P.d * sizeof(float));
  }
  if (out_assign_local) {
    int64_t off = 0;
    for (KmShard* s : shards) {
      VRS_CUDA(cudaSetDevice(s->device));
      if (s->n_local > 0) {
        if (iters > 0)
          VRS_CUDA(cudaMemcpy(out_assign_local + off, s->assign.p, (size_t)s->n_local * sizeof(int32_t),
                              cudaMemcpyDeviceToHost));
        else
          memset(out_assign_local + off, 0, (size_t)s->n_local * sizeof(int32_t));
      }
      off += s->n_local;
    }
  }
  *out_iters = iters;
  *out_inertia = inertia;
  return VRS_OK;
}

}  // namespace

extern "C" {

int vrs_kmeans_fit(const float* x, int64_t n, int32_t d, int32_t k, const float* init,
                   int32_t max_iters, float tol, int32_t metric, int32_t num_gpus,
                   float* out_centroids, int32_t* out_assign, int32_t* out_k, int32_t* out_iters,
                   double* out_inertia) {
  if (!out_k || !out_iters || !out_inertia) return fail(VRS_ERR_INVALID_CONFIG, "null output");
  *out_k = 0;
  *out_iters = 0;
  *out_inertia = 0.0;
  if (num_gpus < 1) return fail(VRS_ERR_INVALID_CONFIG, "num_gpus must be at least 1");
  int avail = available_devices();
  if (num_gpus > avail)
    return fail(VRS_ERR_INSUFFICIENT_DEVICES, "Insufficient hardware GPUs: requested " +
                                                  std::to_string(num_gpus) + " device(s), but only " +
                                                  std::to_string(avail) + " physical GPU(s) found");
  if (d < 1 || n < 0 || k < 0 || max_iters < 0 || !valid_metric(metric))
    return fail(VRS_ERR_INVALID_CONFIG, "bad k-means arguments");
  if (n == 0 || k == 0) return VRS_OK;
  if (!x || !out_centroids) return fail(VRS_ERR_INVALID_CONFIG, "null buffer");
  KmParams P;
  P.n_global = n;
  P.d = d;
  P.dp = round_up(d, 8);
  P.k = (int)std::min<int64_t>(k, n);
  P.max_iters = max_iters;
  P.metric = metric;
  P.tol = tol;
  const int g = (int)std::min<int64_t>(num_gpus, n);
  P.nranks = g;
  P.rank_mode = false;
  std::vector<std::unique_ptr<KmShard>> own;
  std::vector<KmShard*> shards;
  std::vector<ncclComm_t> clique;
  const int64_t chunk = (n + g - 1) / g;
  for (int r = 0; r < g; r++) {
    auto s = std::make_unique<KmShard>();
    s->device = r;
    VRS_CUDA(cudaSetDevice(r));
    VRS_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    int64_t b = std::min(n, r * chunk), e = std::min(n, b + chunk);
    s->n_local = e - b;
    VRS_TRY(km_prepare_shard(P, s.get(), x + b * d, VRS_MEM_HOST));
    shards.push_back(s.get());
    own.push_back(std::move(s));
  }
  if (g > 1) {
    clique.resize(g);
    std::vector<int> devs(g);
    for (int r = 0; r < g; r++) devs[r] = r;
    VRS_NCCL(ncclCommInitAll(clique.data(), g, devs.data()));
    for (int r = 0; r < g; r++) shards[r]->comm = clique[r];
  }
  const float* init_ptr = init ? init : x;  // NULL -> first k' points
  int st = km_run(P, shards, init_ptr, out_centroids, out_assign, out_iters, out_inertia);
  own.clear();
  for (ncclComm_t c : clique) ncclCommDestroy(c);
  if (st == VRS_OK) *out_k = P.k;
  return st;
}

int vrs_kmeans_fit_rank(vrs_comm* comm, const float* x_local, int64_t n_local, int64_t n_global,
                        int32_t d, int32_t k, const float* init, int32_t max_iters, float tol,
                        int32_t metric, int32_t mem, float* out_centroids, int32_t* out_assign,
                        int32_t* out_k, int32_t* out_iters, double* out_inertia) {
  if (!comm || !out_k || !out_iters || !out_inertia) return fail(VRS_ERR_INVALID_CONFIG, "null argument");
  *out_k = 0;
  *out_iters = 0;
  *out_inertia = 0.0;
  if (d < 1 || n_local < 0 || n_global < n_local || k < 0 || max_iters < 0 || !valid_metric(metric) ||
      (mem != VRS_MEM_HOST && mem != VRS_MEM_DEVICE))
    return fail(VRS_ERR_INVALID_CONFIG, "bad k-means arguments");
  if (n_global == 0 || k == 0) return VRS_OK;
  if ((n_local > 0 && !x_local) || !out_centroids) return fail(VRS_ERR_INVALID_CONFIG, "null buffer");
  KmParams P;
  P.n_global = n_global;
  P.d = d;
  P.dp = round_up(d, 8);
  P.k = (int)std::min<int64_t>(k, n_global);
  P.max_iters = max_iters;
  P.metric = metric;
  P.tol = tol;
  P.nranks = comm->nranks;
  P.rank_mode = true;
  auto s = std::make_unique<KmShard>();
  s->device = comm->device;
  s->comm = comm->comm;
  s->n_local = n_local;
  VRS_CUDA(cudaSetDevice(comm->device));
  VRS_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  VRS_TRY(km_prepare_shard(P, s.get(), x_local, mem));
  std::vector<float> init_buf((size_t)P.k * d);
  if (init) {
    memcpy(init_buf.data(), init, init_buf.size() * sizeof(float));
  } else {
    // First k' global rows live on rank 0; broadcast them.
    DBuf tmp;
    VRS_TRY(tmp.reserve(init_buf.size() * sizeof(float)));
    if (comm->rank == 0) {
      if (n_local < P.k) return fail(VRS_ERR_INVALID_CONFIG, "rank 0 holds fewer than k rows; pass init");
      VRS_CUDA(cudaMemcpy2DAsync(tmp.p, d * sizeof(float), s->x.p, P.dp * sizeof(float), d * sizeof(float),
                                 P.k, cudaMemcpyDeviceToDevice, s->stream));
    }
    VRS_NCCL(ncclBroadcast(tmp.p, tmp.p, init_buf.size(), ncclFloat32, 0, s->comm, s->stream));
    VRS_TRY(stream_wait(s->stream, s->comm, env_timeout()));
    VRS_CUDA(cudaMemcpy(init_buf.data(), tmp.p, init_buf.size() * sizeof(float), cudaMemcpyDeviceToHost));
    tmp.release();
  }
  std::vector<KmShard*> shards{s.get()};
  int st = km_run(P, shards, init_buf.data(), out_centroids, out_assign, out_iters, out_inertia);
  if (st == VRS_OK) *out_k = P.k;
  return st;
}

}  // extern "C"
