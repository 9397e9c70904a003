// The extern "C" entry points of include/wdl_b200.h: argument validation (before any launch or write),
// status codes and per-thread error messages, the per-device error word, and the tensor-map encoder.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/wdl_b200.h"
#include "common.cuh"
#include "w4a4_gemm.h"
#include "w4a4_quant.h"

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int ok() {
  g_error.clear();
  return WDL_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

__device__ uint32_t g_device_error;

constexpr int kMaxDevices = 64;
uint32_t* g_error_word[kMaxDevices] = {};

// Address of this device's error word (resolved once per device, with that device current).
uint32_t* error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (!g_error_word[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_error_word[dev] = static_cast<uint32_t*>(p);
  }
  return g_error_word[dev];
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ok();
  return fail(WDL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

namespace wdl {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* elem_strides,
                  CUtensorMapInterleave interleave, CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2,
                  CUtensorMapFloatOOBfill fill) {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return false;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn(map, dtype, rank, base, dims, strides, box, elem_strides, interleave, swizzle, l2, fill) ==
         CUDA_SUCCESS;
}

}  // namespace wdl

extern "C" {

const char* wdl_last_error(void) { return g_error.c_str(); }

const char* wdl_version(void) { return "wdl_b200 0.1 sm_100a"; }

int wdl_device_error(void* stream, uint32_t* code) {
  if (!code) return fail(WDL_ERR_ARGUMENT, "code must not be null");
  *code = 0;
  uint32_t* w = error_word();
  if (!w) return fail(WDL_ERR_CUDA, "cannot resolve the device error word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "cudaStreamSynchronize");
  e = cudaMemcpy(code, w, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "read of the device error word");
  if (*code != 0) {
    const uint32_t zero = 0;
    cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    return fail(WDL_ERR_DEVICE, "a kernel gave up a bounded wait (device error code %u)", *code);
  }
  return ok();
}

static bool valid_codes(int f) { return f == WDL_CODES_INT8 || f == WDL_CODES_E4M3; }

int wdl_w4a4_quantize_rows(const void* x, int x_dtype, int64_t ldx, const uint16_t* smooth, int M, int K,
                           int scale_dtype, int code_format, void* codes, float* scales, uint8_t* packed,
                           void* stream) {
  if (!valid_codes(code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", code_format);
  if (M < 0 || K <= 0 || K % 64 != 0) return fail(WDL_ERR_ARGUMENT, "K must be a positive multiple of 64 (got %d)", K);
  if (x_dtype != WDL_BF16 && x_dtype != WDL_F32) return fail(WDL_ERR_ARGUMENT, "x must be bf16 or f32");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (ldx < K) return fail(WDL_ERR_ARGUMENT, "ldx (%lld) < K (%d)", static_cast<long long>(ldx), K);
  const int64_t esize = x_dtype == WDL_F32 ? 4 : 2;
  if (M == 0) return ok();
  if (!x || !codes || !scales) return fail(WDL_ERR_ARGUMENT, "x, codes and scales must not be null");
  if (!aligned(x, 16) || (ldx * esize) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "x rows must be 16-byte aligned");
  if (!aligned(codes, 8) || !aligned(scales, 4) || (packed && !aligned(packed, 4)) || (smooth && !aligned(smooth, 16)))
    return fail(WDL_ERR_ARGUMENT, "misaligned output or smooth pointer");
  wdl::w4a4::quantize_rows_launch(x, x_dtype, ldx, smooth, M, K, scale_dtype, code_format,
                                  static_cast<int8_t*>(codes), scales, packed, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "quantize_rows launch");
}

int wdl_w4a4_unpack_weight(const uint8_t* qweight, const void* wscales, int scale_dtype, int N, int K,
                           int code_format, void* codes, float* scales, void* stream) {
  if (!valid_codes(code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", code_format);
  if (N <= 0 || K <= 0 || K % 64 != 0) return fail(WDL_ERR_ARGUMENT, "N > 0 and K a positive multiple of 64 required");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (!qweight || !wscales || !codes || !scales) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (!aligned(qweight, 4) || !aligned(codes, 8) || !aligned(wscales, 2) || !aligned(scales, 4))
    return fail(WDL_ERR_ARGUMENT, "misaligned pointer");
  wdl::w4a4::unpack_weight_launch(qweight, static_cast<const uint16_t*>(wscales), scale_dtype, N, K, code_format,
                                  static_cast<int8_t*>(codes), scales, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "unpack_weight launch");
}

static int gemm_common(wdl::w4a4::GemmArgs& a, void* stream) {
  if (!valid_codes(a.code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", a.code_format);
  if (a.M < 0) return fail(WDL_ERR_ARGUMENT, "M must be >= 0");
  if (a.M == 0) return ok();
  if (!a.a || !a.b || !a.wscale || !a.ep.ascale || !a.ep.out) return fail(WDL_ERR_ARGUMENT, "null operand pointer");
  if (!aligned(a.ep.out, 16) || (a.ep.residual && !aligned(a.ep.residual, 16)))
    return fail(WDL_ERR_ARGUMENT, "output and residual must be 16-byte aligned");
  a.err = error_word();
  if (!a.err) return fail(WDL_ERR_CUDA, "cannot resolve the device error word");
  const char* why = "";
  const int st = wdl::w4a4::gemm_launch(a, static_cast<cudaStream_t>(stream), &why);
  if (st == 1) return fail(WDL_ERR_ARGUMENT, "%s", why);
  if (st != 0) return fail(WDL_ERR_CUDA, "%s", why);
  return ok();
}

static void operands(wdl::w4a4::GemmArgs& g, const void* a, const float* a_scales, const void* w, const float* w_scales,
                     int code_format, int M, int N, int K) {
  g.a = static_cast<const int8_t*>(a), g.lda = K, g.b = static_cast<const int8_t*>(w), g.ldb = K;
  g.wscale = w_scales, g.M = M, g.N = N, g.K = K, g.a_signed = 1u, g.code_format = code_format;
  g.ep.ascale = a_scales;
}

int wdl_w4a4_gemm(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                  const float* bias, int M, int N, int K, uint16_t* y, int64_t ldy, void* stream) {
  if (ldy < N || (ldy * 2) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "ldy must be >= N with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  g.ep.mode = wdl::w4a4::kEpiBf16, g.ep.bias = bias, g.ep.out = y, g.ep.ld_out = ldy;
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_residual(const void* a, const float* a_scales, const void* w, const float* w_scales,
                           int code_format, const float* bias, const float* gate, const float* residual, int64_t ldr,
                           int M, int N, int K, float* out, int64_t ldo, void* stream) {
  if (!residual) return fail(WDL_ERR_ARGUMENT, "residual must not be null");
  if (ldr < N || ldo < N || (ldr * 4) % 16 != 0 || (ldo * 4) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "ldr, ldo must be >= N with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  g.ep.mode = wdl::w4a4::kEpiResidualF32, g.ep.bias = bias, g.ep.gate = gate;
  g.ep.residual = residual, g.ep.ld_res = ldr, g.ep.out = out, g.ep.ld_out = ldo;
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_group_partials(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                 int code_format, int M, int N, int K, int group, int32_t* out, int64_t ldo,
                                 void* stream) {
  if (group < 0 || K <= 0 || group >= K / 64) return fail(WDL_ERR_ARGUMENT, "group out of range");
  if (ldo < N || (ldo * 4) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "ldo must be >= N with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  g.ep.mode = wdl::w4a4::kEpiDumpGroup, g.ep.out = out, g.ep.ld_out = ldo, g.ep.dump_group = group;
  return gemm_common(g, stream);
}

size_t wdl_w4a4_linear_workspace(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  const size_t codes = (static_cast<size_t>(M) * K + 255) / 256 * 256;
  const size_t scales = static_cast<size_t>(K / 64) * M * 4;
  return codes + scales;
}

int wdl_w4a4_linear(const uint16_t* x, int64_t ldx, int M, int K, const uint16_t* smooth, int scale_dtype,
                    const void* w, const float* w_scales, int code_format, const float* bias, int N, uint16_t* y,
                    int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0) return fail(WDL_ERR_ARGUMENT, "M must be >= 0");
  if (M == 0) return ok();
  if (K % 128 != 0 || N % 256 != 0) return fail(WDL_ERR_ARGUMENT, "K % 128 == 0 and N % 256 == 0 required");
  if (ldy < N || (ldy * 2) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "ldy must be >= N with 16-byte aligned rows");
  if (!valid_codes(code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", code_format);
  const size_t need = wdl_w4a4_linear_workspace(M, K);
  if (!workspace || workspace_bytes < need)
    return fail(WDL_ERR_ARGUMENT, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  if (!aligned(workspace, 256)) return fail(WDL_ERR_ARGUMENT, "workspace must be 256-byte aligned");
  if (!w || !w_scales) return fail(WDL_ERR_ARGUMENT, "null weight pointer");
  int8_t* codes = static_cast<int8_t*>(workspace);
  float* scales = reinterpret_cast<float*>(static_cast<char*>(workspace) + (static_cast<size_t>(M) * K + 255) / 256 * 256);
  int st = wdl_w4a4_quantize_rows(x, WDL_BF16, ldx, smooth, M, K, scale_dtype, code_format, codes, scales, nullptr,
                                  stream);
  if (st != WDL_OK) return st;
  return wdl_w4a4_gemm(codes, scales, w, w_scales, code_format, bias, M, N, K, y, ldy, stream);
}

}  // extern "C"
