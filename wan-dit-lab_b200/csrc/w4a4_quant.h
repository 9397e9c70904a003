// Internal interface of the INT4 group quantizer and the weight unpacker.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace wdl {
namespace w4a4 {

// x_dtype: 0 bf16, 2 f32. Requirements (checked by the caller): K % 64 == 0, ldx * size and x 16-byte aligned,
// codes 8-byte aligned, packed 4-byte aligned.
// code_format: 0 int8 two's complement, 1 E4M3, 3 float16 codes (two bytes each, 16-byte aligned), 4 prescaled
// float16 values with one power of two per row (CodeFormat in w4a4_gemm.h). err (nullable): the device error word,
// which the prescaled format sets to kErrInexact when a value could not be held exactly.
void quantize_rows_launch(const void* x, int x_dtype, int64_t ldx, const uint16_t* smooth, int M, int K,
                          int scale_dtype, int code_format, int8_t* codes, float* scales, uint8_t* packed,
                          uint32_t* err, cudaStream_t stream);

// N * K % 8 == 0; qweight 4-byte aligned, codes 8-byte aligned.
void unpack_weight_launch(const uint8_t* qweight, const uint16_t* wscales, int scale_dtype, int N, int K,
                          int code_format, int8_t* codes, float* scales, cudaStream_t stream);

// act [M, ld_act] f32 = x [M, ldx] (bf16, or f32 with x_f32) proj_down [K, rank] f32 (lowrank.cu). Requirements
// (checked by the caller): K % 32 == 0, x and its rows 16-byte aligned, rank % 4 == 0, rank <= ld_act.
cudaError_t lowrank_down_launch(const void* x, int x_f32, int64_t ldx, int M, int K, const float* down, int rank,
                                float* act, int64_t ld_act, cudaStream_t s);

}  // namespace w4a4
}  // namespace wdl
