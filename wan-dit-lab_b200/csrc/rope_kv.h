// Internal interface of the RoPE, FP8 KV-store and QKV-preparation kernels.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace wdl {
namespace ropekv {

struct StoreArgs {
  const void* k;  // [B, N, H, D], element strides k_strides
  const void* v;
  int k_dtype, v_dtype;  // 0 bf16, 1 f16, 2 f32
  int64_t k_strides[4], v_strides[4];
  int B, N, H, D;
  uint8_t* cache_k;  // [B, capacity, H, D] e4m3, contiguous
  float* cache_ks;   // [B, capacity, H]
  uint8_t* cache_v;
  float* cache_vs;
  int capacity, at;
};
void store_kv_launch(const StoreArgs& a, cudaStream_t s);

struct RopeArgs {
  const void* x;  // [B, L, H, D], element strides x_strides
  int x_dtype;    // 0 bf16, 1 f16, 2 f32, 3 f64
  int64_t x_strides[4];
  int B, L, H, D;
  int grids[3 * 64];  // (f, h, w) of each sample, B <= 64
  const void* freq;  // [2, P, D/2], element strides f_strides
  int freq_dtype;    // 2 f32, 3 f64
  int64_t f_strides[3];
  int start;
  void* out;  // [B, L, H, D] contiguous
  int out_dtype;
};
void rope_launch(const RopeArgs& a, cudaStream_t s);

struct QkvPrepArgs {
  const __nv_bfloat16* qkv;  // [n, ld_qkv]: q | k | v of dim channels each
  int64_t ld_qkv;
  int n, dim;  // tokens, channels of q in this call (heads * 128)
  const float* norm_q;  // [dim] RMSNorm weights (this call's slice)
  const float* norm_k;
  float eps;
  const float* sumsq;  // [n, 2] sums of squares of q and k over all norm_dim channels (nullable: this call's own)
  int norm_dim;        // channels the RMSNorm averages over (dim unless the heads are split across shards)
  const float* freq;  // [2, P, 64] float32, contiguous
  int64_t freq_table_stride, freq_positions_stride;
  int grid_h, grid_w, start;  // token t: positions (start + t / (h w), t / w % h, t % w)
  float* q_out;  // [n, dim] float32 (rotated, normalized)
  float* k_out;
  uint8_t* cache_k;  // [capacity, heads, 128] e4m3 (nullable: no store)
  float* cache_ks;
  uint8_t* cache_v;
  float* cache_vs;
  int at;
};
void qkv_prep_launch(const QkvPrepArgs& a, cudaStream_t s);

}  // namespace ropekv
}  // namespace wdl
