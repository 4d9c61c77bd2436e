// profile.cu -- optional per-kernel device timing with CUDA events
// (vrs_profile_* in include/vrs.h). Each timed launch records a start and a
// stop event on its own stream; totals are gathered when read.
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "vrs_internal.cuh"

namespace vrs {
namespace {

struct Pending {
  std::string name;
  int device;
  cudaEvent_t start, stop;
};

std::mutex g_mu;
int g_on = 0;  // 0 off, 1 every stage, 2 whole-loop stages only
std::vector<Pending> g_pending;
std::map<std::string, std::pair<double, int64_t>> g_acc;
std::atomic<int64_t> g_launches{0};

void harvest_locked() {
  int prev = 0;
  cudaGetDevice(&prev);
  for (Pending& p : g_pending) {
    cudaSetDevice(p.device);
    cudaEventSynchronize(p.stop);
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
      auto& a = g_acc[p.name];
      a.first += ms;
      a.second += 1;
    }
    cudaEventDestroy(p.start);
    cudaEventDestroy(p.stop);
  }
  g_pending.clear();
  cudaSetDevice(prev);
}

}  // namespace

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void prof_count(const char* name, int64_t n) {
  std::lock_guard<std::mutex> g(g_mu);
  if (g_on != 1) return;
  g_acc[name].second += n;
}

ProfToken prof_begin(const char* name, cudaStream_t s) {
  ProfToken t;
  {
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_on) return t;
    if (g_on == 2 && std::strcmp(name, "kmeans_loop") != 0) return t;
  }
  t.active = true;
  t.name = name;
  cudaGetDevice(&t.device);
  cudaEventCreate(&t.start);
  cudaEventCreate(&t.stop);
  cudaEventRecord(t.start, s);
  return t;
}

void prof_end(ProfToken& t, cudaStream_t s) {
  if (!t.active) return;
  cudaEventRecord(t.stop, s);
  std::lock_guard<std::mutex> g(g_mu);
  g_pending.push_back(Pending{t.name, t.device, t.start, t.stop});
  t.active = false;
}

}  // namespace vrs

extern "C" int vrs_profile_enable(int32_t on) {
  std::lock_guard<std::mutex> g(vrs::g_mu);
  vrs::g_on = on;
  return VRS_OK;
}

extern "C" int vrs_profile_reset(void) {
  std::lock_guard<std::mutex> g(vrs::g_mu);
  vrs::harvest_locked();
  vrs::g_acc.clear();
  vrs::g_launches.store(0);
  return VRS_OK;
}

extern "C" int vrs_profile_read(const char* name, double* total_ms, int64_t* launches) {
  if (!name) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, "null profile name");
    return VRS_ERR_INVALID_CONFIG;
  }
  std::lock_guard<std::mutex> g(vrs::g_mu);
  vrs::harvest_locked();
  if (std::string(name) == "*") {
    if (total_ms) *total_ms = 0.0;
    if (launches) *launches = vrs::g_launches.load();
    return VRS_OK;
  }
  auto it = vrs::g_acc.find(name);
  if (total_ms) *total_ms = it == vrs::g_acc.end() ? 0.0 : it->second.first;
  if (launches) *launches = it == vrs::g_acc.end() ? 0 : it->second.second;
  return VRS_OK;
}
