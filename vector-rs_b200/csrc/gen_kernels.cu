// gen_kernels.cu -- device and host entry points of the seeded generator in
// vrs_gen.cuh. Built with -fmad=false (device) and -ffp-contract=off (host)
// so both produce identical bits.
#include "vrs_gen.cuh"
#include "vrs_internal.cuh"

namespace vrs {
namespace {

__global__ void gen_rows_kernel(int kind, uint64_t seed, uint32_t stream, int64_t row0, int64_t rows,
                                int d, int64_t ld, float* __restrict__ out,
                                const float* __restrict__ centres, uint32_t K, double sigma) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= rows) return;
  vrs_gen::gen_row(kind, seed, stream, row0 + r, d, out + r * ld, centres, K, sigma);
}

}  // namespace

int launch_gen_rows(int kind, uint64_t seed, uint32_t stream, int64_t row0, int64_t rows, int d,
                    int ld, float* out, const float* centres, uint32_t K, double sigma,
                    cudaStream_t s) {
  if (rows <= 0) return VRS_OK;
  gen_rows_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, s>>>(kind, seed, stream, row0, rows, d,
                                                                 ld, out, centres, K, sigma);
  VRS_CUDA(cudaGetLastError());
    count_launch();
  return VRS_OK;
}

}  // namespace vrs

extern "C" int vrs_gen_rows_host(int32_t kind, uint64_t seed, uint32_t stream, int64_t row0,
                                 int64_t rows, int32_t d, int64_t ld, float* out,
                                 const float* centres, uint32_t K, double sigma) {
  if (kind < 0 || kind > 4 || d <= 0 || rows < 0 || ld < d || (kind == 4 && (!centres || K == 0))) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, "vrs_gen_rows_host: bad arguments");
    return VRS_ERR_INVALID_CONFIG;
  }
  for (int64_t r = 0; r < rows; r++)
    vrs_gen::gen_row(kind, seed, stream, row0 + r, d, out + r * ld, centres, K, sigma);
  return VRS_OK;
}

extern "C" int vrs_gen_rows_device(int32_t kind, uint64_t seed, uint32_t stream_id, int64_t row0,
                                   int64_t rows, int32_t d, int64_t ld, float* out,
                                   const float* centres, uint32_t K, double sigma,
                                   void* cuda_stream) {
  if (kind < 0 || kind > 4 || d <= 0 || rows < 0 || ld < d || (kind == 4 && (!centres || K == 0))) {
    vrs::set_error(VRS_ERR_INVALID_CONFIG, "vrs_gen_rows_device: bad arguments");
    return VRS_ERR_INVALID_CONFIG;
  }
  return vrs::launch_gen_rows(kind, seed, stream_id, row0, rows, d, (int)ld, out, centres, K, sigma,
                              (cudaStream_t)cuda_stream);
}
