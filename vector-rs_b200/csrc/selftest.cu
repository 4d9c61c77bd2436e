// selftest.cu -- self-test of the device-side bounded wait.
//
// Every mbarrier wait in the tensor-core kernels goes through tc::mbar_wait,
// which gives up after a time limit, records a stage code in the kernel's
// error word and returns, so a stalled pipeline ends the kernel instead of
// hanging the GPU; the host then reports VRS_ERR_TIMEOUT. This file runs
// that exact helper on an mbarrier that nothing ever arrives on (no TMA copy
// or tensor-core work is in flight), so a test can watch the limit expire
// and the status reach the C ABI, with the context still usable afterwards.
#include "tc_common.cuh"
#include "vrs_internal.cuh"

namespace vrs {
namespace {

constexpr int kSelftestCode = 99;

__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, int* err) {
  __shared__ uint64_t bar;
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);  // one arrival would complete phase 0; none comes
    s_abort = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_wait(&bar, 0, (volatile int*)&s_abort, err, kSelftestCode, limit_ns);
}

}  // namespace
}  // namespace vrs

extern "C" int vrs_selftest_bounded_wait(int64_t limit_ns) {
  using namespace vrs;
  if (limit_ns < 1000 || limit_ns > 1000000000LL) {
    set_error(VRS_ERR_INVALID_CONFIG, "vrs_selftest_bounded_wait: limit must be in [1 us, 1 s]");
    return VRS_ERR_INVALID_CONFIG;
  }
  int* d_err = nullptr;
  VRS_CUDA(cudaMalloc(&d_err, sizeof(int)));
  int h_err = 0;
  cudaError_t e = cudaMemset(d_err, 0, sizeof(int));
  if (e == cudaSuccess) {
    bounded_wait_selftest_kernel<<<1, 32>>>((uint64_t)limit_ns, d_err);
    count_launch();
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d_err);
  if (e != cudaSuccess) {
    set_error(cuda_status(e), std::string("vrs_selftest_bounded_wait: ") + cudaGetErrorString(e));
    return cuda_status(e);
  }
  if (h_err == kSelftestCode) {
    set_error(VRS_ERR_TIMEOUT, "bounded device wait gave up (stage code " + std::to_string(h_err) + ")");
    return VRS_ERR_TIMEOUT;
  }
  set_error(VRS_ERR_DRIVER, "bounded device wait returned without its error code");
  return VRS_ERR_DRIVER;
}
