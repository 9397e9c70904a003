// Internal interface of the W4A4 GEMM and the activation quantizer (not part of the public C-ABI).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace wdl {

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry point (no link to libcuda).
bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* elem_strides,
                  CUtensorMapInterleave interleave, CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2,
                  CUtensorMapFloatOOBfill fill);

namespace w4a4 {

// How the 4-bit integer codes are held, one per byte. Both are exact for codes in [-8, 15]; E4M3 lets the
// tensor core (kind::f8f6f4) leave float32 group partials that need no conversion before promotion.
enum CodeFormat : int {
  kCodesInt8 = 0,  // two's complement int8 (tcgen05 kind::i8, int32 partials)
  kCodesE4M3 = 1,  // the code's value as an FP8 E4M3 number (tcgen05 kind::f8f6f4, fp32 partials)
  // 2 is unused
  kCodesF16Fold = 3,  // float16 operands: activation codes, weights folded with their bf16 group scales and one
                      // power of two 2^-F (w4a4_gemm_fold.cu); the weight "scales" argument is the float 2^F
  kCodesF16Pre = 4,   // float16 activations with their bf16 group scales folded in too: code * sx * 2^-E_m, one
                      // power of two per row (exact: a code has <= 3 significant bits, sx 8); the activation
                      // "scales" are the rows' 2^E_m [M]; weights as kCodesF16Fold. The GEMM accumulates all of K
                      // in TMEM (no per-group promotion); GELU epilogues write the hidden layer in kCodesF16Fold.
};

enum EpilogueMode : int {
  kEpiBf16 = 0,         // out bf16 [M, N] = acc + bias
  kEpiResidualF32 = 1,  // out f32 [M, N] = residual + float(bf16(acc + bias)) * gate (gate optional)
  kEpiDumpGroup = 2,    // out int32 [M, N] = the raw integer partial of group dump_group (debug / parity)
  kEpiGeluU4 = 3,       // out codes [M, N] (E4M3) + out_scales [N / 64, M]: unsigned INT4 of GELU(acc + bias) + shift
};

// The kernels take this block by value as a launch parameter. It is kept within 128 bytes: on B200 the same
// kernels with a 160-byte block (the low-rank fields appended to 64-bit strides) ran their epilogues far slower,
// the GELU-requantizing one 1.5x (FFN-1, M 1392: 176 us against 116 us), with the same registers and no spills;
// packed to 128 bytes they are back at 116 us. Hence 32-bit leading dimensions, range-checked by the callers.
struct GemmEpilogue {
  int mode;
  int dump_group;         // kEpiDumpGroup
  const float* ascale;    // [K / 64, M] activation group scales ([M] row powers of two for kCodesF16Pre)
  const float* bias;      // [N] or null
  const float* gate;      // [N] or null (kEpiResidualF32)
  const float* residual;  // [M, ld_res] f32 (kEpiResidualF32)
  void* out;              // bf16, f32 or int32 per mode, row stride ld_out elements
  float* out_scales;                // kEpiGeluU4: [N / 64, M] group scales of the hidden codes
  const __nv_bfloat16* out_smooth;  // kEpiGeluU4: [N] the next layer's smoothing (nullable)
  const float* addend;  // [M, ld_add] f32 added to the product before bias (the low-rank branch), nullable
  float* gelu_out;  // kEpiGeluU4: [M, ld_gelu] f32 GELU(y) before shift and smoothing (the next low-rank input), nullable
  // The low-rank branch formed in the epilogue instead of an addend: y += lr_act[m, :] . lr_up[n, :] over lr_rank
  // (a multiple of 4): lr_act [M, lr_ld] f32 = x proj_down, lr_up [N, lr_rank] f32 = proj_up. Nullable.
  const float* lr_act;
  const float* lr_up;
  int ld_res, ld_out, ld_add, ld_gelu, lr_ld;  // row strides in elements
  int out_scale_dtype;  // kEpiGeluU4: 0 bf16, 1 f16 rounding of the stored scales
  float gelu_shift;     // kEpiGeluU4: added after GELU (0.171875)
  int lr_rank;
};
static_assert(sizeof(GemmEpilogue) <= 128, "the epilogue parameter block must stay within 128 bytes");

#ifdef __CUDACC__
// Adds row m, columns [n0, n0 + kCount) of the low-rank branch's product into acc (before the bias), when the
// epilogue has one. A separate pass over the finished accumulators keeps the modes' own loops as they are without it.
template <int kCount>
__device__ __forceinline__ void add_addend(const GemmEpilogue& ep, int m, int n0, float* acc) {
  if (!ep.addend) return;
  const float* p = ep.addend + static_cast<size_t>(m) * ep.ld_add + n0;
#pragma unroll
  for (int j = 0; j < kCount; ++j) acc[j] += __ldg(p + j);
}

// Adds row m, columns [n0, n0 + kCount) of the low-rank branch's up-projection into acc (before the bias), when the
// epilogue has one: acc[j] += sum_r lr_act[m, r] lr_up[n0 + j, r], four ranks at a time (one 16-byte load of the
// row's activations, then per column one 16-byte load that every lane of the warp shares and four FMAs).
template <int kCount>
__device__ __forceinline__ void add_lowrank(const GemmEpilogue& ep, int m, int n0, float* acc) {
  if (!ep.lr_act) return;
  const float* act = ep.lr_act + static_cast<size_t>(m) * ep.lr_ld;
  const float* up = ep.lr_up + static_cast<size_t>(n0) * ep.lr_rank;
  for (int r = 0; r < ep.lr_rank; r += 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(act + r));
#pragma unroll
    for (int j = 0; j < kCount; ++j) {
      // loaded where used: hoisted, the loads of all kCount columns would be held in registers at once
      float4 u;
      asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(u.x), "=f"(u.y), "=f"(u.z), "=f"(u.w)
                   : "l"(up + static_cast<size_t>(j) * ep.lr_rank + r));
      acc[j] = fmaf(a.w, u.w, fmaf(a.z, u.z, fmaf(a.y, u.y, fmaf(a.x, u.x, acc[j]))));
    }
  }
}
#endif

struct GemmArgs {
  const int8_t* a;  // [M, lda] activation codes, one per byte
  int64_t lda;      // bytes between rows of a (multiple of 16)
  const int8_t* b;  // [N, ldb] weight codes, one per byte
  int64_t ldb;
  const float* wscale;  // [K / 64, N] weight group scales (the float 2^F for the float16 formats)
  int M, N, K;
  uint32_t a_signed;  // int8 codes: 1 signed, 0 unsigned (the fused MLP's hidden layer)
  int code_format;    // CodeFormat of both operands
  int variant;        // promotion arithmetic: 0 scalar fp32, 1 packed f32x2 (same roundings)
  GemmEpilogue ep;
  uint32_t* err;  // device error word
};

// Validates and launches; returns 0, or a nonzero status with *why set.
// Shape and alignment checks of gemm_launch alone (no CUDA call): 0, or 1 with *why set.
int gemm_validate(const GemmArgs& a, const char** why);
int gemm_launch(const GemmArgs& args, cudaStream_t stream, const char** why);

// The same GEMM for kCodesF16Fold operands (N % 256 == 0, K % 64 == 0; wscale = the float 2^F; no dump mode).
int gemm_fold_validate(const GemmArgs& a, const char** why);
int gemm_fold_launch(const GemmArgs& args, cudaStream_t stream, const char** why);
// w16 [N, K] float16 = code * wscale * 2^-shift from packed codes and bf16 / f16 scales [K / 64, N];
// *inexact (device) counts elements that are not exact normal float16 numbers.
void fold_weight_launch(const uint8_t* qweight, const uint16_t* wscales, int scale_dtype, int N, int K, int shift,
                        uint16_t* w16, unsigned int* inexact, cudaStream_t stream);

}  // namespace w4a4
}  // namespace wdl
