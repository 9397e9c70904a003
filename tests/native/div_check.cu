// Test-only kernel: counts the pairs (x, s) for which the library's div_rn_by(x, s, __frcp_rn(s)) differs in any
// bit from the IEEE quotient __fdiv_rn(x, s). Built by tests/test_division_gpu.py into a scratch directory; the
// library itself never contains it.
#include <cstdint>
#include "common.cuh"

namespace {

__device__ __forceinline__ uint64_t mix(uint64_t z) {  // splitmix64 finalizer
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Pair i of the sweep. mode 0: s a positive float with exponent in [-60, 20], x = s * u for u uniform in
// [-2^20, 2^20] (quotients of every magnitude the quantizers see, and far beyond); mode 1: u = k + 1/2 + d with
// k in [-9, 8] and d a few ulps (the rounding boundaries of INT4 / INT8 codes); mode 2: x, s random bit patterns
// of normal floats with |x / s| in [2^-100, 2^100].
__device__ void pair(uint64_t seed, int mode, uint64_t i, float& x, float& s) {
  const uint64_t a = mix(seed + 2 * i), b = mix(seed + 2 * i + 1);
  if (mode == 2) {
    const uint32_t es = 77 + static_cast<uint32_t>(a % 100), ex = es - 50 + static_cast<uint32_t>(b % 100);
    s = __uint_as_float((es << 23) | static_cast<uint32_t>(a >> 41));
    x = __uint_as_float(((b >> 63) << 31) | (ex << 23) | static_cast<uint32_t>(b >> 41 & 0x7FFFFF));
    return;
  }
  const int e = -60 + static_cast<int>(a % 81);
  s = ldexpf(1.f + static_cast<float>(a >> 40) * 0x1p-24f, e);
  float u;
  if (mode == 0) {
    u = (static_cast<float>(b >> 40) * 0x1p-24f * 2.f - 1.f) * 0x1p20f;
  } else {
    const int k = -9 + static_cast<int>(b % 18);
    const int d = static_cast<int>((b >> 8) % 9) - 4;
    u = __fadd_rn(static_cast<float>(k) + 0.5f, d * ldexpf(1.f, -23 + (k >= 4 || k <= -5 ? 3 : 2)));
  }
  x = __fmul_rn(s, u);
}

__global__ void check_kernel(uint64_t seed, int mode, uint64_t n, unsigned long long* mismatches, float* example) {
  unsigned long long bad = 0;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    float x, s;
    pair(seed, mode, i, x, s);
    const float want = __fdiv_rn(x, s);
    const float got = wdl::div_rn_by(x, s, __frcp_rn(s));
    if (__float_as_uint(want) != __float_as_uint(got)) {
      ++bad;
      example[0] = x, example[1] = s;
    }
  }
  if (bad) atomicAdd(mismatches, bad);
}

}  // namespace

extern "C" int div_check(uint64_t seed, int mode, uint64_t n, unsigned long long* mismatches, float* example) {
  unsigned long long* d_bad = nullptr;
  float* d_ex = nullptr;
  if (cudaMalloc(&d_bad, sizeof(*d_bad)) != cudaSuccess) return 1;
  if (cudaMalloc(&d_ex, 2 * sizeof(float)) != cudaSuccess) return 1;
  cudaMemset(d_bad, 0, sizeof(*d_bad));
  cudaMemset(d_ex, 0, 2 * sizeof(float));
  check_kernel<<<148 * 8, 256>>>(seed, mode, n, d_bad, d_ex);
  const cudaError_t st = cudaDeviceSynchronize();
  cudaMemcpy(mismatches, d_bad, sizeof(*d_bad), cudaMemcpyDeviceToHost);
  cudaMemcpy(example, d_ex, 2 * sizeof(float), cudaMemcpyDeviceToHost);
  cudaFree(d_bad);
  cudaFree(d_ex);
  return st == cudaSuccess ? 0 : 2;
}
