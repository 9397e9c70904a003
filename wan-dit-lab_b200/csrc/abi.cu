// The extern "C" entry points of include/wdl_b200.h: argument validation (before any launch or write),
// status codes and per-thread error messages, the per-device error word, and the tensor-map encoder.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/wdl_b200.h"
#include "common.cuh"
#include "w4a4_gemm.h"
#include "norm_quant.h"
#include "rope_kv.h"
#include "sage.h"
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

int set_last_error(int code, const char* message) {
  g_error = message ? message : "";
  return code;
}

uint32_t* device_error_word() { return error_word(); }

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
    return fail(WDL_ERR_DEVICE, "%s (device error code %u)",
                *code == wdl::kErrIndex     ? "an index map held an entry out of range"
                : *code == wdl::kErrInexact ? "a prescaled (f16pre) operand could not hold a group's values exactly: "
                                              "a group scale lies more than 2^28 below its row's largest (use the "
                                              "e4m3 or f16fold format for this layer)"
                                            : "a kernel gave up a bounded wait",
                *code);
  }
  return ok();
}

static bool valid_codes(int f) {
  return f == WDL_CODES_INT8 || f == WDL_CODES_E4M3 || f == WDL_CODES_F16_FOLD || f == WDL_CODES_F16_PRE;
}

// Bytes of one code in a code format's operand (float16 codes of the folded format take two).
static int code_bytes(int f) { return f == WDL_CODES_F16_FOLD || f == WDL_CODES_F16_PRE ? 2 : 1; }
static bool folded(int f) { return f == WDL_CODES_F16_FOLD || f == WDL_CODES_F16_PRE; }

static bool scales_aligned(const void* p) { return aligned(p, 4); }

int wdl_w4a4_quantize_rows(const void* x, int x_dtype, int64_t ldx, const uint16_t* smooth, int M, int K,
                           int scale_dtype, int code_format, void* codes, float* scales, uint8_t* packed,
                           void* stream) {
  if (!valid_codes(code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", code_format);
  if (M < 0 || K <= 0 || K % 64 != 0) return fail(WDL_ERR_ARGUMENT, "K must be a positive multiple of 64 (got %d)", K);
  if (x_dtype != WDL_BF16 && x_dtype != WDL_F32) return fail(WDL_ERR_ARGUMENT, "x must be bf16 or f32");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (ldx < K) return fail(WDL_ERR_ARGUMENT, "ldx (%lld) < K (%d)", static_cast<long long>(ldx), K);
  if (code_format == WDL_CODES_F16_PRE && (scale_dtype != WDL_BF16 || packed))
    return fail(WDL_ERR_ARGUMENT, "the prescaled format takes bf16 scales (exact products) and no packed copy");
  const int64_t esize = x_dtype == WDL_F32 ? 4 : 2;
  if (M == 0) return ok();
  if (!x || !codes || !scales) return fail(WDL_ERR_ARGUMENT, "x, codes and scales must not be null");
  if (!aligned(x, 16) || (ldx * esize) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "x rows must be 16-byte aligned");
  if (!aligned(codes, 8 * code_bytes(code_format)) || !scales_aligned(scales) ||
      (packed && !aligned(packed, 4)) || (smooth && !aligned(smooth, 16)))
    return fail(WDL_ERR_ARGUMENT, "misaligned output or smooth pointer");
  wdl::w4a4::quantize_rows_launch(x, x_dtype, ldx, smooth, M, K, scale_dtype, code_format,
                                  static_cast<int8_t*>(codes), scales, packed, error_word(),
                                  static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "quantize_rows launch");
}

int wdl_w4a4_unpack_weight(const uint8_t* qweight, const void* wscales, int scale_dtype, int N, int K,
                           int code_format, void* codes, float* scales, void* stream) {
  if (!valid_codes(code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", code_format);
  if (folded(code_format)) return fail(WDL_ERR_ARGUMENT, "folded weights are made by wdl_w4a4_fold_weight");
  if (N <= 0 || K <= 0 || K % 64 != 0) return fail(WDL_ERR_ARGUMENT, "N > 0 and K a positive multiple of 64 required");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (!qweight || !wscales || !codes || !scales) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (!aligned(qweight, 4) || !aligned(codes, 8) || !aligned(wscales, 2) || !scales_aligned(scales))
    return fail(WDL_ERR_ARGUMENT, "misaligned pointer");
  wdl::w4a4::unpack_weight_launch(qweight, static_cast<const uint16_t*>(wscales), scale_dtype, N, K, code_format,
                                  static_cast<int8_t*>(codes), scales, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "unpack_weight launch");
}

int wdl_w4a4_fold_weight(const uint8_t* qweight, const void* wscales, int scale_dtype, int N, int K, int shift,
                         uint16_t* w16, uint32_t* inexact, void* stream) {
  if (N <= 0 || K <= 0 || K % 64 != 0) return fail(WDL_ERR_ARGUMENT, "N > 0 and K a positive multiple of 64 required");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (shift < -100 || shift > 100) return fail(WDL_ERR_ARGUMENT, "shift out of range");
  if (!qweight || !wscales || !w16 || !inexact) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (!aligned(qweight, 4) || !aligned(w16, 16) || !aligned(wscales, 2) || !aligned(inexact, 4))
    return fail(WDL_ERR_ARGUMENT, "misaligned pointer");
  wdl::w4a4::fold_weight_launch(qweight, static_cast<const uint16_t*>(wscales), scale_dtype, N, K, shift, w16,
                                reinterpret_cast<unsigned int*>(inexact), static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "fold_weight launch");
}

static int gemm_common(wdl::w4a4::GemmArgs& a, void* stream) {
  if (!valid_codes(a.code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", a.code_format);
  if (a.M < 0) return fail(WDL_ERR_ARGUMENT, "M must be >= 0");
  if (a.M == 0) return ok();
  if (!a.a || !a.b || !a.wscale || !a.ep.ascale || !a.ep.out) return fail(WDL_ERR_ARGUMENT, "null operand pointer");
  if (!aligned(a.ep.out, 16) || (a.ep.residual && !aligned(a.ep.residual, 16)) || (a.ep.bias && !aligned(a.ep.bias, 16)))
    return fail(WDL_ERR_ARGUMENT, "output, residual and bias must be 16-byte aligned");
  const int f = a.code_format;
  const char* why = "";
  const int v = folded(f) ? wdl::w4a4::gemm_fold_validate(a, &why) : wdl::w4a4::gemm_validate(a, &why);
  if (v != 0) return fail(WDL_ERR_ARGUMENT, "%s", why);
  a.err = error_word();
  if (!a.err) return fail(WDL_ERR_CUDA, "cannot resolve the device error word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int st = folded(f) ? wdl::w4a4::gemm_fold_launch(a, s, &why) : wdl::w4a4::gemm_launch(a, s, &why);
  if (st == 1) return fail(WDL_ERR_ARGUMENT, "%s", why);
  if (st != 0) return fail(WDL_ERR_CUDA, "%s", why);
  return ok();
}

static void operands(wdl::w4a4::GemmArgs& g, const void* a, const float* a_scales, const void* w, const float* w_scales,
                     int code_format, int M, int N, int K) {
  g.a = static_cast<const int8_t*>(a), g.lda = K, g.b = static_cast<const int8_t*>(w), g.ldb = K;
  g.wscale = w_scales, g.M = M, g.N = N, g.K = K, g.a_signed = 1u, g.code_format = code_format;
  static const int variant = [] {
    const char* v = getenv("WDL_GEMM_VARIANT");
    return v ? atoi(v) : 1;  // f32x2 promotion by default (the scalar one needs more registers than it has)
  }();
  g.variant = variant;
  g.ep.ascale = a_scales;
}

// The GEMM epilogue's leading dimensions reach the kernels as 32-bit ints (GemmEpilogue).
static bool ld32(int64_t ld) { return ld <= INT32_MAX; }

// The low-rank branch's fp32 addend [M, ld_add], when given.
static int set_addend(wdl::w4a4::GemmArgs& g, const float* addend, int64_t ld_add, int N) {
  if (!addend) return ok();
  if (ld_add < N || !ld32(ld_add) || !aligned(addend, 4))
    return fail(WDL_ERR_ARGUMENT, "addend rows must hold N floats (ld_add < 2^31)");
  g.ep.addend = addend, g.ep.ld_add = static_cast<int>(ld_add);
  return ok();
}

int wdl_lowrank_down(const void* x, int x_dtype, int64_t ldx, int M, int K, const float* down, int rank, float* act,
                     int64_t ld_act, void* stream) {
  if (M < 0 || K <= 0 || K % 32 != 0) return fail(WDL_ERR_ARGUMENT, "M >= 0 and K a positive multiple of 32 required");
  if (rank <= 0 || rank % 4 != 0) return fail(WDL_ERR_ARGUMENT, "rank must be a positive multiple of 4");
  if (x_dtype != WDL_BF16 && x_dtype != WDL_F32) return fail(WDL_ERR_ARGUMENT, "x must be bf16 or f32");
  const int esize = x_dtype == WDL_F32 ? 4 : 2;
  if (ldx < K || (ldx * esize) % 16 != 0 || ld_act < rank)
    return fail(WDL_ERR_ARGUMENT, "ldx >= K with 16-byte aligned rows and ld_act >= rank required");
  if (M == 0) return ok();
  if (!x || !down || !act || !aligned(x, 16) || !aligned(down, 16)) return fail(WDL_ERR_ARGUMENT, "null or misaligned pointer");
  return cuda_status(wdl::w4a4::lowrank_down_launch(x, x_dtype == WDL_F32, ldx, M, K, down, rank, act, ld_act,
                                                    static_cast<cudaStream_t>(stream)),
                     "lowrank_down launch");
}

// The low-rank branch formed in the epilogue (wdl_lowrank), when given.
static int set_lowrank(wdl::w4a4::GemmArgs& g, const wdl_lowrank* lr) {
  if (!lr) return ok();
  if (!lr->act || !lr->up) return fail(WDL_ERR_ARGUMENT, "low-rank act and up must not be null");
  if (lr->rank <= 0 || lr->rank % 4 != 0 || lr->rank > 1024)
    return fail(WDL_ERR_ARGUMENT, "low-rank rank must be a positive multiple of 4, at most 1024");
  if (lr->ld_act < lr->rank || lr->ld_act % 4 != 0 || !ld32(lr->ld_act) || !aligned(lr->act, 16) || !aligned(lr->up, 16))
    return fail(WDL_ERR_ARGUMENT, "low-rank act rows must hold rank floats, 16-byte aligned (ld_act < 2^31)");
  g.ep.lr_act = lr->act, g.ep.lr_ld = static_cast<int>(lr->ld_act), g.ep.lr_up = lr->up, g.ep.lr_rank = lr->rank;
  return ok();
}

int wdl_w4a4_gemm_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                          const float* bias, const wdl_lowrank* lowrank, int M, int N, int K, uint16_t* y,
                          int64_t ldy, void* stream) {
  if (ldy < N || (ldy * 2) % 16 != 0 || !ld32(ldy))
    return fail(WDL_ERR_ARGUMENT, "ldy must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_lowrank(g, lowrank) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.mode = wdl::w4a4::kEpiBf16, g.ep.bias = bias, g.ep.out = y, g.ep.ld_out = static_cast<int>(ldy);
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_residual_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                   int code_format, const float* bias, const wdl_lowrank* lowrank, const float* gate,
                                   const float* residual, int64_t ldr, int M, int N, int K, float* out, int64_t ldo,
                                   void* stream) {
  if (!residual) return fail(WDL_ERR_ARGUMENT, "residual must not be null");
  if (ldr < N || ldo < N || (ldr * 4) % 16 != 0 || (ldo * 4) % 16 != 0 || !ld32(ldr) || !ld32(ldo))
    return fail(WDL_ERR_ARGUMENT, "ldr, ldo must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_lowrank(g, lowrank) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.mode = wdl::w4a4::kEpiResidualF32, g.ep.bias = bias, g.ep.gate = gate;
  g.ep.residual = residual, g.ep.ld_res = static_cast<int>(ldr), g.ep.out = out, g.ep.ld_out = static_cast<int>(ldo);
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_f32_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales,
                              int code_format, const float* bias, const wdl_lowrank* lowrank, int M, int N, int K,
                              float* out, int64_t ldo, void* stream) {
  if (ldo < N || (ldo * 4) % 16 != 0 || !ld32(ldo))
    return fail(WDL_ERR_ARGUMENT, "ldo must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_lowrank(g, lowrank) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.mode = wdl::w4a4::kEpiResidualF32, g.ep.bias = bias, g.ep.residual = nullptr, g.ep.out = out, g.ep.ld_out = static_cast<int>(ldo);
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_add(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                      const float* bias, const float* addend, int64_t ld_add, int M, int N, int K, uint16_t* y,
                      int64_t ldy, void* stream) {
  if (ldy < N || (ldy * 2) % 16 != 0 || !ld32(ldy))
    return fail(WDL_ERR_ARGUMENT, "ldy must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_addend(g, addend, ld_add, N) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.mode = wdl::w4a4::kEpiBf16, g.ep.bias = bias, g.ep.out = y, g.ep.ld_out = static_cast<int>(ldy);
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                  const float* bias, int M, int N, int K, uint16_t* y, int64_t ldy, void* stream) {
  return wdl_w4a4_gemm_add(a, a_scales, w, w_scales, code_format, bias, nullptr, 0, M, N, K, y, ldy, stream);
}

int wdl_w4a4_gemm_residual(const void* a, const float* a_scales, const void* w, const float* w_scales,
                           int code_format, const float* bias, const float* gate, const float* residual, int64_t ldr,
                           int M, int N, int K, float* out, int64_t ldo, void* stream) {
  return wdl_w4a4_gemm_residual_add(a, a_scales, w, w_scales, code_format, bias, nullptr, 0, gate, residual, ldr, M,
                                    N, K, out, ldo, stream);
}

int wdl_w4a4_gemm_residual_add(const void* a, const float* a_scales, const void* w, const float* w_scales,
                               int code_format, const float* bias, const float* addend, int64_t ld_add,
                               const float* gate, const float* residual, int64_t ldr, int M, int N, int K, float* out,
                               int64_t ldo, void* stream) {
  if (!residual) return fail(WDL_ERR_ARGUMENT, "residual must not be null");
  if (ldr < N || ldo < N || (ldr * 4) % 16 != 0 || (ldo * 4) % 16 != 0 || !ld32(ldr) || !ld32(ldo))
    return fail(WDL_ERR_ARGUMENT, "ldr, ldo must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_addend(g, addend, ld_add, N) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.mode = wdl::w4a4::kEpiResidualF32, g.ep.bias = bias, g.ep.gate = gate;
  g.ep.residual = residual, g.ep.ld_res = static_cast<int>(ldr), g.ep.out = out, g.ep.ld_out = static_cast<int>(ldo);
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_f32(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                      const float* bias, const float* addend, int64_t ld_add, int M, int N, int K, float* out,
                      int64_t ldo, void* stream) {
  if (ldo < N || (ldo * 4) % 16 != 0 || !ld32(ldo))
    return fail(WDL_ERR_ARGUMENT, "ldo must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_addend(g, addend, ld_add, N) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.mode = wdl::w4a4::kEpiResidualF32, g.ep.bias = bias, g.ep.residual = nullptr, g.ep.out = out, g.ep.ld_out = static_cast<int>(ldo);
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_group_partials(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                 int code_format, int M, int N, int K, int group, int32_t* out, int64_t ldo,
                                 void* stream) {
  if (group < 0 || K <= 0 || group >= K / 64) return fail(WDL_ERR_ARGUMENT, "group out of range");
  if (ldo < N || (ldo * 4) % 16 != 0 || !ld32(ldo))
    return fail(WDL_ERR_ARGUMENT, "ldo must be >= N (and < 2^31) with 16-byte aligned rows");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  g.ep.mode = wdl::w4a4::kEpiDumpGroup, g.ep.out = out, g.ep.ld_out = static_cast<int>(ldo), g.ep.dump_group = group;
  return gemm_common(g, stream);
}

int wdl_w4a4_gemm_gelu_u4(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                          const float* bias, const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N,
                          int K, uint8_t* codes, int64_t ldc, float* scales, void* stream) {
  return wdl_w4a4_gemm_gelu_u4_add(a, a_scales, w, w_scales, code_format, bias, nullptr, 0, smooth_next, shift,
                                   scale_dtype, M, N, K, codes, ldc, scales, nullptr, 0, stream);
}

static int gelu_u4_impl(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                        const float* bias, const float* addend, int64_t ld_add, const wdl_lowrank* lowrank,
                        const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N, int K, uint8_t* codes,
                        int64_t ldc, float* scales, float* gelu_out, int64_t ld_gelu, void* stream);

int wdl_w4a4_gemm_gelu_u4_add(const void* a, const float* a_scales, const void* w, const float* w_scales,
                              int code_format, const float* bias, const float* addend, int64_t ld_add,
                              const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N, int K,
                              uint8_t* codes, int64_t ldc, float* scales, float* gelu_out, int64_t ld_gelu,
                              void* stream) {
  return gelu_u4_impl(a, a_scales, w, w_scales, code_format, bias, addend, ld_add, nullptr, smooth_next, shift,
                      scale_dtype, M, N, K, codes, ldc, scales, gelu_out, ld_gelu, stream);
}

int wdl_w4a4_gemm_gelu_u4_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                  int code_format, const float* bias, const wdl_lowrank* lowrank,
                                  const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N, int K,
                                  uint8_t* codes, int64_t ldc, float* scales, float* gelu_out, int64_t ld_gelu,
                                  void* stream) {
  return gelu_u4_impl(a, a_scales, w, w_scales, code_format, bias, nullptr, 0, lowrank, smooth_next, shift,
                      scale_dtype, M, N, K, codes, ldc, scales, gelu_out, ld_gelu, stream);
}

}  // extern "C"

static int gelu_u4_impl(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                        const float* bias, const float* addend, int64_t ld_add, const wdl_lowrank* lowrank,
                        const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N, int K, uint8_t* codes,
                        int64_t ldc, float* scales, float* gelu_out, int64_t ld_gelu, void* stream) {
  if (gelu_out && (ld_gelu < N || !ld32(ld_gelu) || !aligned(gelu_out, 4)))
    return fail(WDL_ERR_ARGUMENT, "gelu_out rows must hold N floats (ld_gelu < 2^31)");
  if (code_format == WDL_CODES_INT8)
    return fail(WDL_ERR_ARGUMENT, "the unsigned hidden codes need an E4M3 or float16 code format");
  if (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) return fail(WDL_ERR_ARGUMENT, "scale dtype must be bf16 or f16");
  if (ldc < N || ldc % 16 != 0 || !ld32(ldc)) return fail(WDL_ERR_ARGUMENT, "ldc must be >= N (and < 2^31) and a multiple of 16");
  if (!aligned(codes, 16)) return fail(WDL_ERR_ARGUMENT, "codes must be 16-byte aligned");
  if (!scales) return fail(WDL_ERR_ARGUMENT, "null scales");
  wdl::w4a4::GemmArgs g{};
  operands(g, a, a_scales, w, w_scales, code_format, M, N, K);
  if (set_addend(g, addend, ld_add, N) != WDL_OK || set_lowrank(g, lowrank) != WDL_OK) return WDL_ERR_ARGUMENT;
  g.ep.gelu_out = gelu_out, g.ep.ld_gelu = static_cast<int>(ld_gelu);
  g.ep.mode = wdl::w4a4::kEpiGeluU4, g.ep.bias = bias, g.ep.out = codes, g.ep.ld_out = static_cast<int>(ldc), g.ep.out_scales = scales;
  g.ep.out_smooth = reinterpret_cast<const __nv_bfloat16*>(smooth_next), g.ep.out_scale_dtype = scale_dtype;
  g.ep.gelu_shift = shift;
  return gemm_common(g, stream);
}


namespace wdl {
// The bf16-output GEMM of a W4A4 linear over the quantized rows `codes` / `scales`, filled as every GEMM entry
// point fills it (the same promotion variant) and checked on the host alone (shapes, alignment, tensor-map
// limits), so that a linear the GEMM would refuse is refused before its quantizer writes anything.
int linear_gemm_args(w4a4::GemmArgs& g, const void* codes, const float* scales, const void* w, const float* w_scales,
                     int code_format, const float* bias, int M, int N, int K, uint16_t* y, int64_t ldy) {
  if (ldy > INT32_MAX) return fail(WDL_ERR_ARGUMENT, "ldy must be < 2^31");
  operands(g, codes, scales, w, w_scales, code_format, M, N, K);
  g.ep.mode = w4a4::kEpiBf16, g.ep.bias = bias, g.ep.out = y, g.ep.ld_out = static_cast<int>(ldy);
  if (!codes || !scales || !w || !w_scales || !y) return fail(WDL_ERR_ARGUMENT, "null operand pointer");
  if (!aligned(y, 16) || (bias && !aligned(bias, 16))) return fail(WDL_ERR_ARGUMENT, "output and bias must be 16-byte aligned");
  const char* why = "";
  const int v = folded(code_format) ? w4a4::gemm_fold_validate(g, &why) : w4a4::gemm_validate(g, &why);
  if (v != 0) return fail(WDL_ERR_ARGUMENT, "%s", why);
  return ok();
}
}  // namespace wdl

extern "C" {

size_t wdl_w4a4_linear_workspace(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  const size_t codes = (static_cast<size_t>(M) * K * 2 + 255) / 256 * 256;  // room for float16 codes
  const size_t scales = static_cast<size_t>(K / 64) * M * 4;
  return codes + scales;
}

int wdl_w4a4_linear(const uint16_t* x, int64_t ldx, int M, int K, const uint16_t* smooth, int scale_dtype,
                    const void* w, const float* w_scales, int code_format, const float* bias, int N, uint16_t* y,
                    int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0) return fail(WDL_ERR_ARGUMENT, "M must be >= 0");
  if (M == 0) return ok();
  if (K % 128 != 0 || N % 256 != 0) return fail(WDL_ERR_ARGUMENT, "K % 128 == 0 and N % 256 == 0 required");
  if (ldy < N || (ldy * 2) % 16 != 0 || !ld32(ldy))
    return fail(WDL_ERR_ARGUMENT, "ldy must be >= N (and < 2^31) with 16-byte aligned rows");
  if (!valid_codes(code_format)) return fail(WDL_ERR_ARGUMENT, "unknown code format %d", code_format);
  const size_t need = wdl_w4a4_linear_workspace(M, K);
  if (!workspace || workspace_bytes < need)
    return fail(WDL_ERR_ARGUMENT, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  if (!aligned(workspace, 256)) return fail(WDL_ERR_ARGUMENT, "workspace must be 256-byte aligned");
  if (!w || !w_scales) return fail(WDL_ERR_ARGUMENT, "null weight pointer");
  int8_t* codes = static_cast<int8_t*>(workspace);
  float* scales = reinterpret_cast<float*>(static_cast<char*>(workspace) + (static_cast<size_t>(M) * K * 2 + 255) / 256 * 256);
  wdl::w4a4::GemmArgs g{};
  int st = wdl::linear_gemm_args(g, codes, scales, w, w_scales, code_format, bias, M, N, K, y, ldy);
  if (st != WDL_OK) return st;
  st = wdl_w4a4_quantize_rows(x, WDL_BF16, ldx, smooth, M, K, scale_dtype, code_format, codes, scales, nullptr, stream);
  if (st != WDL_OK) return st;
  return gemm_common(g, stream);
}

int wdl_store_kv_fp8(const void* k, int k_dtype, const int64_t* k_strides, const void* v, int v_dtype,
                     const int64_t* v_strides, int B, int N, int H, int D, uint8_t* cache_k, float* cache_ks,
                     uint8_t* cache_v, float* cache_vs, int capacity, int at, void* stream) {
  if (B < 0 || N < 0 || H < 0 || D < 1) return fail(WDL_ERR_ARGUMENT, "K and V must have matching [B,N,H,D] shapes");
  for (int dt : {k_dtype, v_dtype})
    if (dt != WDL_BF16 && dt != WDL_F16 && dt != WDL_F32) return fail(WDL_ERR_ARGUMENT, "K and V must be FP16, BF16 or FP32");
  if (at < 0 || at + N > capacity) return fail(WDL_ERR_ARGUMENT, "Write exceeds cache bounds");
  if (!k_strides || !v_strides) return fail(WDL_ERR_ARGUMENT, "strides must not be null");
  for (int i = 0; i < 4; ++i)
    if (k_strides[i] < 0 || v_strides[i] < 0) return fail(WDL_ERR_ARGUMENT, "strides must be nonnegative");
  if (static_cast<int64_t>(B) * N * H == 0) return ok();
  if (!k || !v || !cache_k || !cache_ks || !cache_v || !cache_vs) return fail(WDL_ERR_ARGUMENT, "null pointer");
  wdl::ropekv::StoreArgs a{};
  a.k = k, a.v = v, a.k_dtype = k_dtype, a.v_dtype = v_dtype;
  for (int i = 0; i < 4; ++i) a.k_strides[i] = k_strides[i], a.v_strides[i] = v_strides[i];
  a.B = B, a.N = N, a.H = H, a.D = D, a.cache_k = cache_k, a.cache_ks = cache_ks, a.cache_v = cache_v;
  a.cache_vs = cache_vs, a.capacity = capacity, a.at = at;
  wdl::ropekv::store_kv_launch(a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "store_kv_fp8 launch");
}

int wdl_rope_apply(const void* x, int x_dtype, const int64_t* x_strides, int B, int L, int H, int D, const int* grids,
                   const void* freq, int freq_dtype, const int64_t* freq_strides, int positions, int start, void* out,
                   int out_dtype, void* stream) {
  if (x_dtype < 0 || x_dtype > 3 || out_dtype < 0 || out_dtype > 3)
    return fail(WDL_ERR_ARGUMENT, "Floating input and output dtypes required");
  if (freq_dtype != WDL_F32 && freq_dtype != 3) return fail(WDL_ERR_ARGUMENT, "Floating input and real FP32/FP64 frequencies required");
  if (B < 1 || L < 0 || H < 0 || D < 2 || D % 2) return fail(WDL_ERR_ARGUMENT, "Input must be (batch, token, heads, even dim)");
  if (B > 64) return fail(WDL_ERR_ARGUMENT, "at most 64 samples per call");
  if (start < 0) return fail(WDL_ERR_ARGUMENT, "start_frame must be a nonnegative integer");
  if (!grids || !x_strides || !freq_strides) return fail(WDL_ERR_ARGUMENT, "null metadata");
  const int spatial = (D / 2) / 3;
  for (int b = 0; b < B; ++b) {
    const int f = grids[3 * b], h = grids[3 * b + 1], w = grids[3 * b + 2];
    if (f < 0 || h <= 0 || w <= 0 || static_cast<int64_t>(f) * h * w > L)
      return fail(WDL_ERR_ARGUMENT, "Grid exceeds sequence length or has invalid dimensions");
    if (start + f > positions || (spatial && (h > positions || w > positions)))
      return fail(WDL_ERR_ARGUMENT, "Grid or offset exceeds frequency bounds");
  }
  if (static_cast<int64_t>(L) * H == 0) return ok();
  if (!x || !freq || !out) return fail(WDL_ERR_ARGUMENT, "null pointer");
  wdl::ropekv::RopeArgs a{};
  a.x = x, a.x_dtype = x_dtype, a.B = B, a.L = L, a.H = H, a.D = D, a.freq = freq, a.freq_dtype = freq_dtype;
  for (int i = 0; i < 4; ++i) a.x_strides[i] = x_strides[i];
  for (int i = 0; i < 3; ++i) a.f_strides[i] = freq_strides[i];
  for (int i = 0; i < 3 * B; ++i) a.grids[i] = grids[i];
  a.start = start, a.out = out, a.out_dtype = out_dtype;
  wdl::ropekv::rope_launch(a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "rope launch");
}

int wdl_qkv_prep(const uint16_t* qkv, int64_t ld, int n, int dim, const float* norm_q, const float* norm_k, float eps,
                 const float* freq, int positions, int grid_h, int grid_w, int start, float* q_out, float* k_out,
                 uint8_t* cache_k, float* cache_ks, uint8_t* cache_v, float* cache_vs, int capacity, int at,
                 void* stream) {
  if (dim != 1024 && dim != 2048 && dim != 3072 && dim != 4096)
    return fail(WDL_ERR_ARGUMENT, "dim must be 1024, 2048, 3072 or 4096 (heads of 128)");
  return wdl_qkv_prep_sharded(qkv, ld, n, dim, norm_q, norm_k, eps, nullptr, dim, freq, positions, grid_h, grid_w,
                              start, q_out, k_out, cache_k, cache_ks, cache_v, cache_vs, capacity, at, stream);
}

int wdl_qkv_prep_sharded(const uint16_t* qkv, int64_t ld, int n, int dim, const float* norm_q, const float* norm_k,
                         float eps, const float* sumsq, int norm_dim, const float* freq, int positions, int grid_h,
                         int grid_w, int start, float* q_out, float* k_out, uint8_t* cache_k, float* cache_ks,
                         uint8_t* cache_v, float* cache_vs, int capacity, int at, void* stream) {
  if (dim <= 0 || dim % 128 != 0 || dim > 4096) return fail(WDL_ERR_ARGUMENT, "dim must be a multiple of 128 (heads), at most 4096");
  if (sumsq ? norm_dim < dim : norm_dim != dim)
    return fail(WDL_ERR_ARGUMENT, "norm_dim must be dim, or (with sumsq) the channels of all shards");
  if (n < 0 || ld < 3 * dim || (ld * 2) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "qkv rows must hold 3 dim channels, 16-byte aligned");
  if (grid_h <= 0 || grid_w <= 0 || n % (grid_h * grid_w) != 0)
    return fail(WDL_ERR_ARGUMENT, "n must be a whole number of frames of grid_h x grid_w tokens");
  if (start < 0 || start + n / (grid_h * grid_w) > positions || grid_h > positions || grid_w > positions)
    return fail(WDL_ERR_ARGUMENT, "Grid or offset exceeds frequency bounds");
  if (cache_k && (at < 0 || at + n > capacity)) return fail(WDL_ERR_ARGUMENT, "Write exceeds cache bounds");
  if (n == 0) return ok();
  if (!qkv || !norm_q || !norm_k || !freq || !q_out || !k_out) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (cache_k && (!cache_ks || !cache_v || !cache_vs)) return fail(WDL_ERR_ARGUMENT, "null cache pointer");
  if (!aligned(qkv, 16) || !aligned(q_out, 16) || !aligned(k_out, 16) || !aligned(sumsq, 8) ||
      (cache_k && (!aligned(cache_k, 8) || !aligned(cache_v, 8))))
    return fail(WDL_ERR_ARGUMENT, "misaligned pointer");
  wdl::ropekv::QkvPrepArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv), a.ld_qkv = ld, a.n = n, a.dim = dim, a.norm_q = norm_q;
  a.norm_k = norm_k, a.eps = eps, a.sumsq = sumsq, a.norm_dim = norm_dim, a.freq = freq;
  a.freq_table_stride = static_cast<int64_t>(positions) * 64;
  a.freq_positions_stride = 64, a.grid_h = grid_h, a.grid_w = grid_w, a.start = start, a.q_out = q_out;
  a.k_out = k_out, a.cache_k = cache_k, a.cache_ks = cache_ks, a.cache_v = cache_v, a.cache_vs = cache_vs, a.at = at;
  wdl::ropekv::qkv_prep_launch(a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "qkv_prep launch");
}

int wdl_ln_quant(const void* x, int x_dtype, int64_t ldx, int M, int K, float eps, const float* ln_w,
                 const float* ln_b, int round_ln_bf16, const float* mod_shift, const float* mod_scale,
                 const uint16_t* smooth, int scale_dtype, int code_format, void* codes, float* scales, void* stream) {
  return wdl_ln_quant_keep(x, x_dtype, ldx, M, K, eps, ln_w, ln_b, round_ln_bf16, mod_shift, mod_scale, smooth,
                           scale_dtype, code_format, codes, scales, nullptr, 0, stream);
}

int wdl_ln_quant_keep(const void* x, int x_dtype, int64_t ldx, int M, int K, float eps, const float* ln_w,
                      const float* ln_b, int round_ln_bf16, const float* mod_shift, const float* mod_scale,
                      const uint16_t* smooth, int scale_dtype, int code_format, void* codes, float* scales,
                      uint16_t* x_out, int64_t ld_xo, void* stream) {
  if (x_dtype != WDL_F32 && x_dtype != WDL_BF16) return fail(WDL_ERR_ARGUMENT, "x must be float32 or bf16");
  if (K <= 0 || K % 256 != 0 || K > 4096) return fail(WDL_ERR_ARGUMENT, "K must be a multiple of 256, at most 4096");
  if (M < 0 || ldx < K) return fail(WDL_ERR_ARGUMENT, "M >= 0 and ldx >= K required");
  if ((ldx * (x_dtype == WDL_F32 ? 4 : 2)) % 16 != 0 || !aligned(x, 16)) return fail(WDL_ERR_ARGUMENT, "x rows must be 16-byte aligned");
  if ((ln_w == nullptr) != (ln_b == nullptr) || (mod_shift == nullptr) != (mod_scale == nullptr))
    return fail(WDL_ERR_ARGUMENT, "affine weight / bias and modulation shift / scale come in pairs");
  if (!valid_codes(code_format) || (scale_dtype != WDL_BF16 && scale_dtype != WDL_F16) ||
      (code_format == WDL_CODES_F16_PRE && scale_dtype != WDL_BF16))
    return fail(WDL_ERR_ARGUMENT, "invalid code format or scale dtype (the prescaled format takes bf16 scales)");
  if (M == 0) return ok();
  if (!codes || !scales || !aligned(codes, 8 * code_bytes(code_format)) || !scales_aligned(scales))
    return fail(WDL_ERR_ARGUMENT, "null or misaligned output");
  if (!aligned(ln_w, 16) || !aligned(ln_b, 16) || !aligned(mod_shift, 16) || !aligned(mod_scale, 16) ||
      !aligned(smooth, 16))
    return fail(WDL_ERR_ARGUMENT, "ln_w, ln_b, mod_shift, mod_scale and smooth must be 16-byte aligned");
  if (x_out && (ld_xo < K || (ld_xo * 2) % 16 != 0 || !aligned(x_out, 16)))
    return fail(WDL_ERR_ARGUMENT, "x_out rows must hold K bf16 channels, 16-byte aligned");
  wdl::norm::LnQuantArgs a{};
  a.x = x, a.x_f32 = x_dtype == WDL_F32, a.ldx = ldx, a.M = M, a.K = K, a.eps = eps, a.ln_w = ln_w, a.ln_b = ln_b;
  a.round_ln_bf16 = round_ln_bf16, a.mod_shift = mod_shift, a.mod_scale = mod_scale;
  a.smooth = reinterpret_cast<const __nv_bfloat16*>(smooth), a.scale_dtype = scale_dtype, a.code_format = code_format;
  a.codes = static_cast<uint8_t*>(codes), a.scales = scales;
  a.x_out = reinterpret_cast<__nv_bfloat16*>(x_out), a.ld_xo = ld_xo;
  a.err = error_word();
  wdl::norm::ln_quant_launch(a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "ln_quant launch");
}

int wdl_rms_rows(const uint16_t* x, int64_t ldx, int M, int K, const float* w, float eps, float* out, int64_t ldo,
                 void* stream) {
  if (K <= 0 || K % 256 != 0 || K > 4096) return fail(WDL_ERR_ARGUMENT, "K must be a multiple of 256, at most 4096");
  return wdl_rms_rows_sharded(x, ldx, M, K, w, eps, nullptr, K, out, ldo, stream);
}

int wdl_rms_rows_sharded(const uint16_t* x, int64_t ldx, int M, int K, const float* w, float eps, const float* sumsq,
                         int norm_dim, float* out, int64_t ldo, void* stream) {
  if (K <= 0 || K % 128 != 0 || K > 4096) return fail(WDL_ERR_ARGUMENT, "K must be a multiple of 128, at most 4096");
  if (sumsq ? norm_dim < K : norm_dim != K)
    return fail(WDL_ERR_ARGUMENT, "norm_dim must be K, or (with sumsq) the channels of all shards");
  if (M < 0 || ldx < K || ldo < K || (ldx * 2) % 16 != 0 || (ldo * 4) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "row strides must hold K channels, 16-byte aligned");
  if (M == 0) return ok();
  if (!x || !w || !out || !aligned(x, 16) || !aligned(out, 16) || !aligned(w, 16) || !aligned(sumsq, 4))
    return fail(WDL_ERR_ARGUMENT, "null or misaligned pointer");
  wdl::norm::rms_rows_launch(reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K, w, eps, sumsq, norm_dim, out, ldo,
                             static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "rms_rows launch");
}

int wdl_rows_sumsq(const uint16_t* x, int64_t ldx, int M, int K, int parts, int64_t part_stride, float* out,
                   void* stream) {
  if (K <= 0 || K % 8 != 0 || K > 4096) return fail(WDL_ERR_ARGUMENT, "K must be a multiple of 8, at most 4096");
  if (parts < 1 || part_stride < 0 || (parts > 1 && part_stride < K) || (part_stride * 2) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "parts >= 1 slices of K channels, 16-byte aligned, not overlapping");
  if (M < 0 || ldx < (parts - 1) * part_stride + K || (ldx * 2) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "rows must hold every slice, 16-byte aligned");
  if (M == 0) return ok();
  if (!x || !out || !aligned(x, 16) || !aligned(out, 4)) return fail(WDL_ERR_ARGUMENT, "null or misaligned pointer");
  wdl::norm::rows_sumsq_launch(reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K, parts, part_stride, out,
                               static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "rows_sumsq launch");
}

int wdl_residual_update(const float* partial, int64_t ldp, const float* bias, const float* gate, float* x, int64_t ldx,
                        int M, int N, void* stream) {
  if (M < 0 || N <= 0 || N % 4 != 0) return fail(WDL_ERR_ARGUMENT, "M >= 0 and N a positive multiple of 4 required");
  if (ldp < N || ldx < N || (ldp * 4) % 16 != 0 || (ldx * 4) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "ldp, ldx must be >= N with 16-byte aligned rows");
  if (M == 0) return ok();
  if (!partial || !x || !aligned(partial, 16) || !aligned(x, 16) || !aligned(bias, 4) || !aligned(gate, 4))
    return fail(WDL_ERR_ARGUMENT, "null or misaligned pointer");
  wdl::norm::residual_update_launch(partial, ldp, bias, gate, x, ldx, M, N, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "residual_update launch");
}

int wdl_modulation(const float* time_in, const float* modulation, int blocks, int dim, float* out, void* stream) {
  if (blocks <= 0 || dim <= 0) return fail(WDL_ERR_ARGUMENT, "blocks and dim must be positive");
  if (!time_in || !modulation || !out) return fail(WDL_ERR_ARGUMENT, "null pointer");
  wdl::norm::modulation_launch(time_in, modulation, blocks, dim, out, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "modulation launch");
}

// The Sage quantizers read four channels at a time: cache rows from 4-byte aligned bases, chunk rows of float32
// from 16-byte aligned bases (bf16: 8-byte), row strides a multiple of 4 elements.
static bool sage_sources_aligned(const uint8_t* cache_k, const uint8_t* cache_v, int at, const void* k, int k_dtype,
                                 int64_t ld_k, const void* v, int v_dtype, int64_t ld_v, int n) {
  if (at > 0 && (!aligned(cache_k, 4) || !aligned(cache_v, 4))) return false;
  if (n <= 0) return true;
  return aligned(k, k_dtype == WDL_F32 ? 16 : 8) && aligned(v, v_dtype == WDL_F32 ? 16 : 8) && ld_k % 4 == 0 &&
         ld_v % 4 == 0;
}

int wdl_sage_prep_kv(const uint8_t* cache_k, const float* cache_ks, const uint8_t* cache_v, const float* cache_vs,
                     int at, const void* k, int k_dtype, int64_t ld_k, const void* v, int v_dtype, int64_t ld_v, int n,
                     int H, int8_t* k_i8, float* k_scale, uint8_t* v_f8, float* v_scale, void* work, size_t work_bytes,
                     void* stream) {
  if (n < 0 || at < 0 || H <= 0 || at + n <= 0) return fail(WDL_ERR_ARGUMENT, "H and L = at + n must be positive");
  if ((k_dtype != WDL_F32 && k_dtype != WDL_BF16) || (v_dtype != WDL_F32 && v_dtype != WDL_BF16))
    return fail(WDL_ERR_ARGUMENT, "chunk K and V must be float32 or bf16");
  if (n > 0 && (ld_k < static_cast<int64_t>(H) * 128 || ld_v < static_cast<int64_t>(H) * 128))
    return fail(WDL_ERR_ARGUMENT, "row strides must hold H x 128 channels");
  if (at > 0 && (!cache_k || !cache_ks || !cache_v || !cache_vs)) return fail(WDL_ERR_ARGUMENT, "null cache pointer");
  if ((n > 0 && (!k || !v)) || !k_i8 || !k_scale || !v_f8 || !v_scale) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (!work || work_bytes < wdl::sage::prep_workspace_floats(at + n, H) * sizeof(float))
    return fail(WDL_ERR_ARGUMENT, "workspace too small");
  if (!sage_sources_aligned(cache_k, cache_v, at, k, k_dtype, ld_k, v, v_dtype, ld_v, n) || !aligned(k_i8, 16) ||
      !aligned(v_f8, 16) || !aligned(v_scale, 16))
    return fail(WDL_ERR_ARGUMENT, "misaligned K / V source or output");
  wdl::sage::PrepArgs a{};
  a.cache_k = cache_k, a.cache_ks = cache_ks, a.cache_v = cache_v, a.cache_vs = cache_vs, a.at = at;
  a.k_chunk = k, a.ld_k = ld_k, a.k_bf16 = k_dtype == WDL_BF16, a.v_chunk = v, a.ld_v = ld_v, a.v_bf16 = v_dtype == WDL_BF16;
  a.n = n, a.H = H, a.k_i8 = k_i8, a.k_scale = k_scale, a.v_f8 = v_f8, a.v_scale = v_scale;
  a.work = static_cast<float*>(work);
  wdl::sage::prep_kv_launch(a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "sage kv prep launch");
}

int wdl_sage_quant_q(const float* q, int64_t ld_q, int nq, int H, int8_t* q_i8, float* q_scale, void* stream) {
  if (nq <= 0 || H <= 0 || ld_q < static_cast<int64_t>(H) * 128) return fail(WDL_ERR_ARGUMENT, "invalid Q shape");
  if (!q || !q_i8 || !q_scale || !aligned(q_i8, 8) || !aligned(q, 16) || ld_q % 4 != 0)
    return fail(WDL_ERR_ARGUMENT, "null or misaligned pointer (q 16-byte aligned, ld_q a multiple of 4)");
  wdl::sage::quant_q_launch(q, ld_q, nq, H, q_i8, q_scale, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "sage quant_q launch");
}

size_t wdl_sage_prep_workspace(int L, int H) {
  if (L <= 0 || H <= 0) return 0;
  return wdl::sage::prep_workspace_floats(L, H) * sizeof(float);
}

static size_t pad128(int x) { return (static_cast<size_t>(x) + 127) / 128 * 128; }
static size_t up256(size_t x) { return (x + 255) / 256 * 256; }

}  // extern "C"

// Forcing-KV's index maps of a Sage call (null: none).
struct SageMaps {
  int cache_rows, cache_heads;
  const int32_t* heads;
  const int32_t* tokens;
};

// Per-token V of wdl_sage_attend (sage.h, PrepArgs::token_v): keys [0, rows0) read in place from the cache, the
// rest from `rows`; each key's scale into tok_scale [H][Lpad], each head's largest into head_max [H].
struct SageTokenV {
  int rows0;
  uint8_t* rows;
  float* tok_scale;
  float* head_max;
};

static int sage_prep_impl(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                          const uint8_t* cache_v, const float* cache_vs, int at, const void* k, int k_dtype,
                          int64_t ld_k, const void* v, int v_dtype, int64_t ld_v, int n, int H, int8_t* q_i8,
                          float* q_scale, int8_t* k_i8, float* k_scale, uint8_t* v_f8, float* v_scale, void* work,
                          size_t work_bytes, const SageMaps* maps, const SageTokenV* tv, void* stream) {
  if (nq <= 0 || n < 0 || at < 0 || H <= 0 || at + n <= 0) return fail(WDL_ERR_ARGUMENT, "nq, H and L = at + n must be positive");
  const bool v_in_cache = tv && !v;  // the chunk's values already in the cache at rows [at, at + n)
  if (v_in_cache) {
    if (maps || tv->rows0 != at + n) return fail(WDL_ERR_ARGUMENT, "the chunk's values are required with index maps");
    v_dtype = WDL_BF16, ld_v = static_cast<int64_t>(H) * 128;
  }
  if ((k_dtype != WDL_F32 && k_dtype != WDL_BF16) || (v_dtype != WDL_F32 && v_dtype != WDL_BF16))
    return fail(WDL_ERR_ARGUMENT, "chunk K and V must be float32 or bf16");
  if (ld_q < static_cast<int64_t>(H) * 128 || (n > 0 && (ld_k < static_cast<int64_t>(H) * 128 || ld_v < static_cast<int64_t>(H) * 128)))
    return fail(WDL_ERR_ARGUMENT, "row strides must hold H x 128 channels");
  if (at > 0 && (!cache_k || !cache_ks || !cache_v || !cache_vs)) return fail(WDL_ERR_ARGUMENT, "null cache pointer");
  if (v_in_cache && n > 0 && (!cache_v || !cache_vs)) return fail(WDL_ERR_ARGUMENT, "null cache pointer");
  if (!q || (n > 0 && (!k || (!v && !v_in_cache))) || !q_i8 || !q_scale || !k_i8 || !k_scale ||
      (!tv && (!v_f8 || !v_scale)) || (tv && (!tv->rows || !tv->tok_scale || !tv->head_max)))
    return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (!work || work_bytes < wdl_sage_prep_workspace(at + n, H))
    return fail(WDL_ERR_ARGUMENT, "workspace of %zu bytes required", wdl_sage_prep_workspace(at + n, H));
  if (!aligned(q_i8, 16) || !aligned(k_i8, 16) || (!tv && (!aligned(v_f8, 16) || !aligned(v_scale, 16))) ||
      !aligned(q, 16) || ld_q % 4 != 0 ||
      !sage_sources_aligned(cache_k, cache_v, at, k, k_dtype, ld_k, v, v_dtype, ld_v, n) ||
      (tv && (!aligned(tv->rows, 16) || !aligned(tv->tok_scale, 16) || (tv->rows0 > 0 && !aligned(cache_v, 16)))))
    return fail(WDL_ERR_ARGUMENT, "misaligned input or output");
  wdl::sage::PrepArgs a{};
  a.cache_k = cache_k, a.cache_ks = cache_ks, a.cache_v = cache_v, a.cache_vs = cache_vs, a.at = at;
  a.k_chunk = k, a.ld_k = ld_k, a.k_bf16 = k_dtype == WDL_BF16, a.v_chunk = v, a.ld_v = ld_v, a.v_bf16 = v_dtype == WDL_BF16;
  a.n = n, a.H = H, a.q = q, a.ld_q = ld_q, a.nq = nq, a.q_i8 = q_i8, a.q_scale = q_scale, a.k_i8 = k_i8;
  a.k_scale = k_scale, a.v_f8 = v_f8, a.v_scale = v_scale, a.work = static_cast<float*>(work);
  if (tv) {
    a.token_v = 1, a.rows0 = tv->rows0, a.v_rows = tv->rows, a.v_tok_scale = tv->tok_scale;
    a.v_head_max = tv->head_max;
  }
  if (maps) {
    a.cache_H = maps->cache_heads, a.cache_rows = maps->cache_rows, a.hmap = maps->heads, a.tmap = maps->tokens;
    a.err = error_word();
    if (!a.err) return fail(WDL_ERR_CUDA, "cannot resolve the device error word");
  }
  wdl::sage::prep_launch(a, static_cast<cudaStream_t>(stream));
  return cuda_status(cudaGetLastError(), "sage prep launch");
}

extern "C" {

int wdl_sage_prep(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                  const uint8_t* cache_v, const float* cache_vs, int at, const void* k, int k_dtype, int64_t ld_k,
                  const void* v, int v_dtype, int64_t ld_v, int n, int H, int8_t* q_i8, float* q_scale, int8_t* k_i8,
                  float* k_scale, uint8_t* v_f8, float* v_scale, void* work, size_t work_bytes, void* stream) {
  return sage_prep_impl(q, ld_q, nq, cache_k, cache_ks, cache_v, cache_vs, at, k, k_dtype, ld_k, v, v_dtype, ld_v, n,
                        H, q_i8, q_scale, k_i8, k_scale, v_f8, v_scale, work, work_bytes, nullptr, nullptr, stream);
}

int wdl_sage_attention(const int8_t* q_i8, const float* q_scale, const int8_t* k_i8, const float* k_scale,
                       const uint8_t* v_f8, const float* v_scale, int nq, int L, int H, float sm_scale, uint16_t* out,
                       int64_t ld_out, void* stream) {
  if (nq <= 0 || L <= 0 || H <= 0) return fail(WDL_ERR_ARGUMENT, "nq, L and H must be positive");
  if (ld_out < static_cast<int64_t>(H) * 128 || (ld_out * 2) % 16 != 0) return fail(WDL_ERR_ARGUMENT, "ld_out must hold H x 128 channels, 16-byte rows");
  if (!q_i8 || !q_scale || !k_i8 || !k_scale || !v_f8 || !v_scale || !out) return fail(WDL_ERR_ARGUMENT, "null pointer");
  if (!aligned(q_i8, 16) || !aligned(k_i8, 16) || !aligned(v_f8, 16) || !aligned(out, 16))
    return fail(WDL_ERR_ARGUMENT, "misaligned pointer");
  uint32_t* err = error_word();
  if (!err) return fail(WDL_ERR_CUDA, "cannot resolve the device error word");
  wdl::sage::AttnArgs a{};
  a.q_i8 = q_i8, a.q_scale = q_scale, a.k_i8 = k_i8, a.k_scale = k_scale, a.v_f8 = v_f8, a.v_scale = v_scale;
  a.nq = nq, a.L = L, a.H = H, a.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  a.out = reinterpret_cast<__nv_bfloat16*>(out), a.ld_out = ld_out;
  const char* why = "";
  const int st = wdl::sage::attn_launch(a, err, static_cast<cudaStream_t>(stream), &why);
  if (st != 0) return fail(WDL_ERR_CUDA, "%s", why);
  return ok();
}

size_t wdl_sage_attend_workspace(int nq, int L, int H) {
  if (nq <= 0 || L <= 0 || H <= 0) return 0;
  const size_t np = pad128(nq), lp = pad128(L), h = static_cast<size_t>(H);
  return up256(h * np * 128) + up256(h * np / 32 * 8 * 4) + up256(h * lp * 128) + up256(h * lp / 64 * 4 * 4) +
         up256(lp * h * 128) + up256(h * lp * 4) + up256(h * 4) + up256(wdl_sage_prep_workspace(L, H));
}

}  // extern "C"

static int sage_attend_impl(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                            const uint8_t* cache_v, const float* cache_vs, int at, const void* k, int k_dtype,
                            int64_t ld_k, const void* v, int v_dtype, int64_t ld_v, int n, int H, float sm_scale,
                            uint16_t* out, int64_t ld_out, void* workspace, size_t workspace_bytes,
                            const SageMaps* maps, void* stream) {
  const int L = at + n;
  if (nq <= 0 || L <= 0 || H <= 0) return fail(WDL_ERR_ARGUMENT, "nq, H and L = at + n must be positive");
  const size_t need = wdl_sage_attend_workspace(nq, L, H);
  if (!workspace || workspace_bytes < need) return fail(WDL_ERR_ARGUMENT, "workspace of %zu bytes required", need);
  if (!aligned(workspace, 256)) return fail(WDL_ERR_ARGUMENT, "workspace must be 256-byte aligned");
  const size_t np = pad128(nq), lp = pad128(L), h = static_cast<size_t>(H);
  char* p = static_cast<char*>(workspace);
  int8_t* q_i8 = reinterpret_cast<int8_t*>(p);
  p += up256(h * np * 128);
  float* q_scale = reinterpret_cast<float*>(p);
  p += up256(h * np / 32 * 8 * 4);
  int8_t* k_i8 = reinterpret_cast<int8_t*>(p);
  p += up256(h * lp * 128);
  float* k_scale = reinterpret_cast<float*>(p);
  p += up256(h * lp / 64 * 4 * 4);
  // V as the cache holds it: keys [0, rows0) in place; the rest (the cached keys of the tile that holds `at`,
  // and the chunk's) in the scratch rows. With maps every key goes through the scratch; with the chunk's values
  // already in the cache (v null) none does.
  SageTokenV tv{};
  tv.rows0 = maps ? 0 : (v ? at / 128 * 128 : L);
  tv.rows = reinterpret_cast<uint8_t*>(p);
  p += up256(lp * h * 128);
  tv.tok_scale = reinterpret_cast<float*>(p);
  p += up256(h * lp * 4);
  tv.head_max = reinterpret_cast<float*>(p);
  p += up256(h * 4);
  if (ld_out < static_cast<int64_t>(H) * 128 || (ld_out * 2) % 16 != 0)
    return fail(WDL_ERR_ARGUMENT, "ld_out must hold H x 128 channels, 16-byte rows");
  if (!out || !aligned(out, 16)) return fail(WDL_ERR_ARGUMENT, "null or misaligned output");
  int st = sage_prep_impl(q, ld_q, nq, cache_k, cache_ks, cache_v, cache_vs, at, k, k_dtype, ld_k, v, v_dtype, ld_v,
                          n, H, q_i8, q_scale, k_i8, k_scale, nullptr, nullptr, p, wdl_sage_prep_workspace(L, H), maps,
                          &tv, stream);
  if (st != WDL_OK) return st;
  uint32_t* err = error_word();
  if (!err) return fail(WDL_ERR_CUDA, "cannot resolve the device error word");
  wdl::sage::AttnArgs a{};
  a.q_i8 = q_i8, a.q_scale = q_scale, a.k_i8 = k_i8, a.k_scale = k_scale;
  a.token_v = 1, a.v_rows0 = cache_v, a.ld_v0 = static_cast<int64_t>(H) * 128, a.rows0 = tv.rows0;
  a.v_rows1 = tv.rows, a.v_tok_scale = tv.tok_scale, a.v_head_max = tv.head_max;
  a.nq = nq, a.L = L, a.H = H, a.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  a.out = reinterpret_cast<__nv_bfloat16*>(out), a.ld_out = ld_out;
  const char* why = "";
  st = wdl::sage::attn_launch(a, err, static_cast<cudaStream_t>(stream), &why);
  if (st != 0) return fail(WDL_ERR_CUDA, "%s", why);
  return ok();
}

extern "C" {

int wdl_sage_attend(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                    const uint8_t* cache_v, const float* cache_vs, int at, const void* k, int k_dtype, int64_t ld_k,
                    const void* v, int v_dtype, int64_t ld_v, int n, int H, float sm_scale, uint16_t* out,
                    int64_t ld_out, void* workspace, size_t workspace_bytes, void* stream) {
  return sage_attend_impl(q, ld_q, nq, cache_k, cache_ks, cache_v, cache_vs, at, k, k_dtype, ld_k, v, v_dtype, ld_v, n,
                          H, sm_scale, out, ld_out, workspace, workspace_bytes, nullptr, stream);
}

int wdl_sage_attend_maps(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                         const uint8_t* cache_v, const float* cache_vs, int cache_rows, int cache_heads,
                         const int32_t* heads, const int32_t* tokens, int at, const void* k, int k_dtype, int64_t ld_k,
                         const void* v, int v_dtype, int64_t ld_v, int n, int H, float sm_scale, uint16_t* out,
                         int64_t ld_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (cache_rows < 0 || cache_heads <= 0) return fail(WDL_ERR_ARGUMENT, "cache_rows >= 0 and cache_heads > 0 required");
  if (!heads && cache_heads != H) return fail(WDL_ERR_ARGUMENT, "without a head map the cache holds the call's H heads");
  if (!tokens && at > cache_rows) return fail(WDL_ERR_ARGUMENT, "without a token map at must not exceed cache_rows");
  if (!aligned(heads, 4) || !aligned(tokens, 4)) return fail(WDL_ERR_ARGUMENT, "misaligned map");
  const SageMaps maps{cache_rows, cache_heads, heads, tokens};
  return sage_attend_impl(q, ld_q, nq, cache_k, cache_ks, cache_v, cache_vs, at, k, k_dtype, ld_k, v, v_dtype, ld_v, n,
                          H, sm_scale, out, ld_out, workspace, workspace_bytes, &maps, stream);
}

}  // extern "C"
