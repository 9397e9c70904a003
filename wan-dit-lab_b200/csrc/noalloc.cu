// wdl_w4a4_linear_noalloc: the W4A4 linear for callers that cannot allocate device memory.
//
// wdl_w4a4_linear needs scratch for the activation's INT4 codes and group scales between its two kernels, and
// takes it from the caller. Some callers have no allocator to take it from, or must not use one on their
// hot path: a native host that drives the model through the C ABI with a fixed device-memory budget (weights
// and KV caches fill the card, so an allocation in the middle of a stream may fail), or a render / streaming
// loop for which cudaMalloc and cudaFree are off limits because they can synchronize the whole device and
// stall every in-flight frame. For them this entry point keeps its scratch in a fixed array of this library's
// own device memory, declared below, and calls no allocator at all.
//
// The array is WDL_W4A4_LINEAR_NOALLOC_MAX_BYTES (16 MiB) per device: enough for M * K * (1 + 1/16) bytes of codes and scales,
// e.g. 1392 tokens x 3072 channels (4.5 MB) or 2640 x 3072 (8.6 MB); larger calls are rejected. Every device
// that loads this library holds the array until the process exits. All calls on a device share it and it
// keeps the last call's contents; nothing in it needs to start at zero (the quantizer writes every code and
// scale the GEMM reads). Two calls whose execution overlaps on the GPU (different streams, no ordering
// between them) race on the array and may corrupt each other's result: order them on one stream or with events.
//
// The host cannot use the array's name as a device address (in host code it names a host-side stand-in). The
// device address is resolved with cudaGetSymbolAddress on the first call on each device, with that device
// current, and kept; that first call should therefore be made before any stream capture begins.
#include "../../include/wdl_b200.h"
#include "common.cuh"
#include "w4a4_gemm.h"
#include "w4a4_quant.h"

namespace wdl {
// Defined in abi.cu (C++ linkage, not part of the C ABI): the per-thread message of wdl_last_error, the device
// error word of the current device that bounded waits report into, and the host-side GEMM set-up.
int set_last_error(int code, const char* message);
uint32_t* device_error_word();
// The bf16-output GEMM of a linear, filled and checked on the host as wdl_w4a4_linear does (abi.cu).
int linear_gemm_args(w4a4::GemmArgs& g, const void* codes, const float* scales, const void* w, const float* w_scales,
                     int code_format, const float* bias, int M, int N, int K, uint16_t* y, int64_t ldy);
}  // namespace wdl

namespace {

constexpr size_t kScratchBytes = WDL_W4A4_LINEAR_NOALLOC_MAX_BYTES;
static __device__ __align__(256) uint8_t g_linear_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};

int fail(int code, const char* msg) { return wdl::set_last_error(code, msg); }

// The device address of the scratch array on the current device: resolved with cudaGetSymbolAddress on the
// first call on each device (with that device current) and kept.
int scratch_address(void** scratch) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(WDL_ERR_CUDA, "wdl_w4a4_linear_noalloc: no usable current device");
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess || !p) return fail(WDL_ERR_CUDA, "wdl_w4a4_linear_noalloc: cudaGetSymbolAddress of the scratch failed");
    g_scratch_addr[dev] = p;
  }
  *scratch = g_scratch_addr[dev];
  return WDL_OK;
}

}  // namespace

extern "C" {

int wdl_w4a4_linear_noalloc(const uint16_t* x, int64_t ldx, int M, int K, const uint16_t* smooth, int scale_dtype,
                            const void* w, const float* w_scales, int code_format, const float* bias, int N,
                            uint16_t* y, int64_t ldy, void* stream) {
  if (M < 0) return fail(WDL_ERR_ARGUMENT, "M must be >= 0");
  if (M == 0) return wdl::set_last_error(WDL_OK, "");
  if (K <= 0 || K % 128 != 0 || N <= 0 || N % 256 != 0)
    return fail(WDL_ERR_ARGUMENT, "K % 128 == 0 and N % 256 == 0 required");
  if (code_format != WDL_CODES_INT8 && code_format != WDL_CODES_E4M3)
    return fail(WDL_ERR_ARGUMENT, "unknown code format (the float16 formats are not supported here)");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (ldx < K || (ldx * 2) % 16 != 0 || ldy < N || (ldy * 2) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "ldx >= K and ldy >= N with 16-byte aligned rows required");
  if (!x || !w || !w_scales || !y) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15)
    return fail(WDL_ERR_ARGUMENT, "x, w and y must be 16-byte aligned");
  // the quantizer reads smooth 16 bytes at a time
  if (smooth && (reinterpret_cast<uintptr_t>(smooth) & 15)) return fail(WDL_ERR_ARGUMENT, "smooth must be 16-byte aligned");
  const size_t codes_bytes = (static_cast<size_t>(M) * K + 255) / 256 * 256;
  const size_t need = codes_bytes + static_cast<size_t>(K / 64) * M * sizeof(float);
  if (need > kScratchBytes)
    return fail(WDL_ERR_ARGUMENT,
                "wdl_w4a4_linear_noalloc: M * K too large for its fixed 16 MiB scratch (needs M * K * 17 / 16 bytes); "
                "use wdl_w4a4_linear with a caller workspace");
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != WDL_OK) return st;
  int8_t* codes = static_cast<int8_t*>(scratch);
  float* scales = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + codes_bytes);
  // the GEMM is filled as wdl_w4a4_linear fills it and checked on the host before anything is launched: a call it
  // would refuse leaves the shared scratch untouched
  wdl::w4a4::GemmArgs g{};
  int gs = wdl::linear_gemm_args(g, codes, scales, w, w_scales, code_format, bias, M, N, K, y, ldy);
  if (gs != WDL_OK) return gs;
  g.err = wdl::device_error_word();
  if (!g.err) return fail(WDL_ERR_CUDA, "wdl_w4a4_linear_noalloc: cannot resolve the device error word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  wdl::w4a4::quantize_rows_launch(x, WDL_BF16, ldx, smooth, M, K, scale_dtype, code_format, codes, scales, nullptr,
                                  g.err, s);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(WDL_ERR_CUDA, "wdl_w4a4_linear_noalloc: quantizer launch failed");
  const char* why = "";
  gs = wdl::w4a4::gemm_launch(g, s, &why);
  if (gs == 1) return fail(WDL_ERR_ARGUMENT, why);
  if (gs != 0) return fail(WDL_ERR_CUDA, why);
  return wdl::set_last_error(WDL_OK, "");
}

}  // extern "C"
