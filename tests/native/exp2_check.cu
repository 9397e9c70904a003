// Test-only kernel: evaluates the library's FMA-pipe 2^x (exp2_fma, csrc/common.cuh) and CUDA's exp2f on the same
// arguments, so that a test can hold the polynomial to its error bound against exact powers of two. Built by
// tests/test_exp2_gpu.py into a scratch directory; the library itself never contains it.
#include <cstdint>
#include "common.cuh"

namespace {

__global__ void exp2_kernel(const float* x, float* poly, float* ref, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    poly[i] = wdl::exp2_fma(x[i]);
    ref[i] = exp2f(x[i]);
  }
}

}  // namespace

// x, poly and ref are device arrays of n floats. Returns 0, or the CUDA error code of the launch or the sync.
extern "C" int exp2_check(const float* x, float* poly, float* ref, int64_t n) {
  exp2_kernel<<<296, 256>>>(x, poly, ref, n);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e;
}
