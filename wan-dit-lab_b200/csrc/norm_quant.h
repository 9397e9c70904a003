// Internal interface of the fused normalization kernels.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace wdl {
namespace norm {

struct LnQuantArgs {
  const void* x;  // [M, ldx] residual stream, float32 (x_f32) or bf16
  int x_f32;
  int64_t ldx;
  int M, K;  // K % 256 == 0, K <= 4096
  float eps;
  const float* ln_w;  // [K] affine weight / bias (nullable: no affine)
  const float* ln_b;
  int round_ln_bf16;       // LayerNorm's result rounded to bf16 (the stream is bf16)
  const float* mod_shift;  // [K] (nullable: no modulation)
  const float* mod_scale;  // [K]
  const __nv_bfloat16* smooth;  // [K] (nullable)
  int scale_dtype;  // 0 bf16, 1 f16
  int code_format;  // 0 int8, 1 e4m3, 3 float16 codes, 4 prescaled float16
  uint8_t* codes;   // [M, K] (two bytes per code in format 3)
  float* scales;    // [K / 64, M] (the rows' powers of two [M] in format 4)
  __nv_bfloat16* x_out;  // [M, ld_xo]: the layer's bf16 input before smoothing (nullable; a low-rank branch reads it)
  int64_t ld_xo;
  uint32_t* err;  // device error word (nullable): format 4 records kErrInexact for a value it could not hold exactly
};
void ln_quant_launch(const LnQuantArgs& a, cudaStream_t s);

void rms_rows_launch(const __nv_bfloat16* x, int64_t ldx, int M, int K, const float* w, float eps, const float* sumsq,
                     int norm_dim, float* out, int64_t ldo, cudaStream_t s);
void rows_sumsq_launch(const __nv_bfloat16* x, int64_t ldx, int M, int K, int parts, int64_t part_stride, float* out,
                       cudaStream_t s);
void residual_update_launch(const float* partial, int64_t ldp, const float* bias, const float* gate, float* x,
                            int64_t ldx, int M, int N, cudaStream_t s);

void modulation_launch(const float* time_in, const float* modulation, int blocks, int dim, float* out, cudaStream_t s);

}  // namespace norm
}  // namespace wdl
