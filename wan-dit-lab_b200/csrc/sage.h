// Internal interface of the SageAttention quantizers (sage.cu) and the attention kernel (sage_attn.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace wdl {

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* elem_strides,
                  CUtensorMapInterleave interleave, CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2,
                  CUtensorMapFloatOOBfill fill);

namespace sage {

struct PrepArgs {
  const uint8_t* cache_k;  // [cap, H, 128] e4m3, tokens [0, at)
  const float* cache_ks;   // [cap, H]
  const uint8_t* cache_v;
  const float* cache_vs;
  int at;
  const void* k_chunk;  // [n, ld_k] float32 or bf16 (k_bf16), head h at column h * 128: tokens [at, at + n)
  int64_t ld_k;
  int k_bf16;
  const void* v_chunk;  // [n, ld_v] float32 or bf16 (v_bf16)
  int64_t ld_v;
  int v_bf16;
  int n, H;
  const float* q;  // [nq, ld_q] float32
  int64_t ld_q;
  int nq;
  int8_t* q_i8;  // [H, npad, 128]
  float* q_scale;  // [H, npad / 32 * 8]
  int8_t* k_i8;  // [H, Lpad, 128]
  float* k_scale;  // [H, Lpad / 64 * 4]
  uint8_t* v_f8;   // [H, 128, Lpad]
  float* v_scale;  // [H, 128]
  float* work;     // prep_workspace_floats(L, H) floats
  // Forcing-KV maps (all optional): the cache holds cache_H heads per row (0: H) and cache_rows rows; head h is
  // cache head hmap[h], cached key j is cache row tmap[j]. err: the device error word (out-of-range entries).
  int cache_H, cache_rows;
  const int* hmap;
  const int* tmap;
  uint32_t* err;
  // Per-token V (token_v != 0, wdl_sage_attend): V keeps the cache's E4M3 rows and per-(token, head) scales
  // instead of v_f8 / v_scale. Keys [0, rows0) are read in place from the cache (rows0 % 128 == 0 or rows0 == L;
  // rows0 is 0 with maps); keys [rows0, L) go to v_rows (row r = key rows0 + r, pitch H * 128 bytes): cached
  // rows copied, the chunk's rows quantized per (token, head) by the cache's own rule. v_chunk null: the chunk's
  // values are already in the cache at rows [at, L) (then rows0 == L).
  int token_v;
  int rows0;
  uint8_t* v_rows;
  float* v_tok_scale;  // [H][Lpad]: each key's scale, 0 past L
  float* v_head_max;   // [H]: the largest of a head's key scales
};
void prep_launch(const PrepArgs& a, cudaStream_t s);     // K / V then Q
void prep_kv_launch(const PrepArgs& a, cudaStream_t s);  // K / V only (q fields unused)
void quant_q_launch(const float* q, int64_t ld_q, int nq, int H, int8_t* q_i8, float* q_scale, cudaStream_t s);
size_t prep_workspace_floats(int L, int H);

struct AttnArgs {
  const int8_t* q_i8;
  const float* q_scale;
  const int8_t* k_i8;
  const float* k_scale;
  const uint8_t* v_f8;   // per-channel V (token_v 0): [H][128][Lpad] E4M3, scales v_scale [H][128]
  const float* v_scale;
  int token_v;  // per-token V: E4M3 rows, keys [0, rows0) at v_rows0 (pitch ld_v0 bytes, head h at byte h * 128),
                // keys [rows0, L) at v_rows1 (pitch H * 128); scales v_tok_scale [H][Lpad], v_head_max [H]
  const uint8_t* v_rows0;
  int64_t ld_v0;
  int rows0;
  const uint8_t* v_rows1;
  const float* v_tok_scale;
  const float* v_head_max;
  int nq, L, H;
  float sm_scale_log2;  // sm_scale * log2(e)
  __nv_bfloat16* out;   // [nq, ld_out] bf16, head h at column h * 128
  int64_t ld_out;
};
int attn_launch(const AttnArgs& a, uint32_t* err, cudaStream_t s, const char** why);

}  // namespace sage
}  // namespace wdl
