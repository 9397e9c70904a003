// Test-only kernel: a bounded wait that nothing ever satisfies. One CTA initialises an mbarrier that expects one
// arrival and waits on its first phase with the library's own mbar_wait (csrc/common.cuh) and a limit given as a
// kernel argument; no thread ever arrives, so every wait must give up after the limit, record its code in the
// library's device error word (the word wdl_device_error reads and clears) and return. Built by
// tests/test_wait_limit_gpu.py into a scratch directory and linked against libwdl_b200.so for the error word's
// address; the library itself never contains it.
#include <cstdint>
#include "common.cuh"

namespace wdl {
uint32_t* device_error_word();  // libwdl_b200.so: the current device's error word
}

namespace {

__global__ void wait_kernel(uint64_t limit_ns, uint32_t code, uint32_t* err, uint32_t* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    wdl::mbar_init(&bar, 1);
    wdl::fence_barrier_init();
  }
  __syncthreads();
  const bool done = wdl::mbar_wait(&bar, 0, err, code, limit_ns);  // nobody arrives on `bar`
  if (!done) atomicAdd(gave_up, 1u);
}

}  // namespace

// Runs the kernel with `threads` waiting threads; *gave_up counts the waits that returned false, *ms is the
// kernel's duration. Returns 0, or the CUDA error code of the first call that failed.
extern "C" int wait_check(uint64_t limit_ns, uint32_t code, int threads, uint32_t* gave_up, float* ms) {
  uint32_t* err = wdl::device_error_word();
  if (!err) return -1;
  uint32_t* count = nullptr;
  cudaError_t e = cudaMalloc(&count, sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  cudaEvent_t t0, t1;
  cudaEventCreate(&t0);
  cudaEventCreate(&t1);
  cudaMemset(count, 0, sizeof(uint32_t));
  cudaEventRecord(t0);
  wait_kernel<<<1, threads>>>(limit_ns, code, err, count);
  cudaEventRecord(t1);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaEventSynchronize(t1);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, t0, t1);
  if (e == cudaSuccess) e = cudaMemcpy(gave_up, count, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  cudaFree(count);
  return e;
}
