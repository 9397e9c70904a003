// SageAttention over the FP8 KV cache on sm_100a: the quantization of Q, K and V as SageAttention 2 defines it
// (read straight from the FP8 cache for the cached tokens, from the chunk's own float keys / bf16 values for
// the rest), and the attention itself on tcgen05 tensor cores: INT8 Q K^T (kind::i8) into TMEM, online softmax
// in registers (one thread per query row), P in FP8 E4M3 times the per-channel-scaled FP8 V (kind::f8f6f4)
// accumulated in TMEM.
//
// Reference: src/wan_dit_lab/kernels/sage_kv.py (the quantizers :29-124 and the call of SageAttention's
// kernel :137-176) and generation/causal.py:193-220 (KVCache.attend). The quantization arithmetic follows the
// reference exactly (see sage_prep below); the layouts are this kernel's own:
//   q_i8  [H][npad][128]   q_scale [H][npad / 32 * 8]   (token t: scale (t / 32) * 8 + t % 8)
//   k_i8  [H][Lpad][128]   k_scale [H][Lpad / 64 * 4]   (key j: scale (j / 64) * 4 + (j % 8) / 2)
//   v_f8  [H][128][Lpad]   v_scale [H][128]             (keys contiguous: the K-major B operand of P V)
// with npad, Lpad multiples of 128 and zero codes in the padding.
#include "common.cuh"
#include "sage.h"

namespace wdl {
namespace sage {

__device__ __forceinline__ uint8_t e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float e4m3_value(uint8_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return __half2float(__half(h));
}

// Token j of head h, channel d, as _load of sage_kv.py:29-40 reads it: the cache byte times its scale before
// `at`, the chunk's value after.
struct Source {
  const uint8_t* cache;  // [cap, H, 128]
  const float* scale;    // [cap, H]
  const void* chunk;     // [n, ld] float32 (keys) or bf16 (values), head h at column h * 128
  int64_t ld;
  int chunk_bf16;
  int at, L, H;
  __device__ __forceinline__ float get(int j, int h, int d) const {
    if (j < at) return e4m3_value(cache[(static_cast<int64_t>(j) * H + h) * 128 + d]) * scale[static_cast<int64_t>(j) * H + h];
    const int64_t off = static_cast<int64_t>(j - at) * ld + h * 128 + d;
    return chunk_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(chunk)[off]) : static_cast<const float*>(chunk)[off];
  }
};

// ---- pass 1: per (64-token tile, head), per channel: sum of K and max |V| over the tile (thread = channel)
__global__ void __launch_bounds__(128) partials_kernel(Source ks, Source vs, float* ksum, float* vmax) {
  const int tile = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  float s = 0.f, m = 0.f;
  const int j0 = tile * 64, j1 = min(ks.L, j0 + 64);
  for (int j = j0; j < j1; ++j) {
    s += ks.get(j, h, d);
    m = fmaxf(m, fabsf(vs.get(j, h, d)));
  }
  ksum[(static_cast<int64_t>(tile) * ks.H + h) * 128 + d] = s;
  vmax[(static_cast<int64_t>(tile) * ks.H + h) * 128 + d] = m;
}

// ---- pass 2: per head: key mean (sum / L) and the V channel scales max(max|V|, 1e-8) / 2.25 (V_MAX, :24)
__global__ void __launch_bounds__(128) reduce_kernel(const float* ksum, const float* vmax, int tiles, int H, int L,
                                                     float* kmean, float* v_scale) {
  const int h = blockIdx.x, d = threadIdx.x;
  float s = 0.f, m = 0.f;
  for (int t = 0; t < tiles; ++t) {
    s += ksum[(static_cast<int64_t>(t) * H + h) * 128 + d];
    m = fmaxf(m, vmax[(static_cast<int64_t>(t) * H + h) * 128 + d]);
  }
  kmean[h * 128 + d] = __fdiv_rn(s, static_cast<float>(L));
  v_scale[h * 128 + d] = __fdiv_rn(fmaxf(m, 1e-8f), 2.25f);
}

// ---- pass 3: K - mean to INT8 and V to FP8, per (64-key block, head). 128 threads.
// K (_quant_k, sage_kv.py:60-85): warp g holds the 16 keys 8 i + 2 g, 8 i + 2 g + 1 (i = 0..7) of the block,
// lane l channels 4 l .. 4 l + 3; scale = max|x| / 127 + 1e-7 over the 16 x 128 values; code = trunc(x / scale
// + 0.5 sign(x)). V (_quant_v, :89-105): thread = channel d, V / v_scale[d] rounded to E4M3, stored transposed.
__global__ void __launch_bounds__(128) quant_kv_kernel(Source ks, Source vs, const float* kmean, const float* v_scale,
                                                       int Lpad, int8_t* k_i8, float* k_scale, uint8_t* v_f8) {
  const int blk = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = ks.L;
  {
    const int g = warp;
    float mean[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) mean[c] = kmean[h * 128 + lane * 4 + c];
    float x[16][4];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = blk * 64 + 8 * i + 2 * g + e;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float v = j < L ? __fsub_rn(ks.get(j, h, lane * 4 + c), mean[c]) : 0.f;
          x[2 * i + e][c] = v;
          amax = fmaxf(amax, fabsf(v));
        }
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = blk * 64 + 8 * i + 2 * g + e;
        uint32_t packed = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float y = __fdiv_rn(x[2 * i + e][c], scale);
          const int q = j < L ? static_cast<int>(truncf(__fadd_rn(y, y >= 0.f ? 0.5f : -0.5f))) : 0;
          packed |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * c);
        }
        *reinterpret_cast<uint32_t*>(k_i8 + (static_cast<int64_t>(h) * Lpad + j) * 128 + lane * 4) = packed;
      }
    if (lane == 0) k_scale[static_cast<int64_t>(h) * (Lpad / 64) * 4 + blk * 4 + g] = scale;
  }
  {
    const int d = threadIdx.x;
    const float s = v_scale[h * 128 + d];
    uint8_t* row = v_f8 + (static_cast<int64_t>(h) * 128 + d) * Lpad + blk * 64;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int j = blk * 64 + q * 16 + k * 4 + b;
          const uint8_t byte = j < L ? e4m3(__fdiv_rn(vs.get(j, h, d), s)) : 0;
          word |= static_cast<uint32_t>(byte) << (8 * b);
        }
        w[k] = word;
      }
      *reinterpret_cast<uint4*>(row + q * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ---- Q to INT8 (quant_q, sage_kv.py:112-124), per (32-token block, head). 128 threads: thread (l, c) with
// l = tid / 16 the lane group (tokens l, l + 8, l + 16, l + 24), c = tid % 16 the channels 8 c .. 8 c + 7.
__global__ void __launch_bounds__(128) quant_q_kernel(const float* q, int64_t ldq, int n, int npad, int8_t* q_i8,
                                                      float* q_scale) {
  const int blk = blockIdx.x, h = blockIdx.y;
  const int l = threadIdx.x >> 4, c = threadIdx.x & 15;
  float x[4][8];
  float amax = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = blk * 32 + r * 8 + l;
    const float* src = q + static_cast<int64_t>(t) * ldq + h * 128 + c * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[r][i] = t < n ? src[i] : 0.f;
      amax = fmaxf(amax, fabsf(x[r][i]));
    }
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = blk * 32 + r * 8 + l;
    uint32_t w[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = __fdiv_rn(x[r][i], scale);
      const int qv = static_cast<int>(truncf(__fadd_rn(y, y >= 0.f ? 0.5f : -0.5f)));
      w[i / 4] |= (static_cast<uint32_t>(qv) & 0xFFu) << (8 * (i % 4));
    }
    *reinterpret_cast<uint2*>(q_i8 + (static_cast<int64_t>(h) * npad + t) * 128 + c * 8) = make_uint2(w[0], w[1]);
  }
  if (c == 0) q_scale[static_cast<int64_t>(h) * (npad / 32) * 8 + blk * 8 + l] = scale;
}

void prep_kv_launch(const PrepArgs& a, cudaStream_t s) {
  const int L = a.at + a.n;
  Source ks{a.cache_k, a.cache_ks, a.k_chunk, a.ld_k, a.k_bf16, a.at, L, a.H};
  Source vs{a.cache_v, a.cache_vs, a.v_chunk, a.ld_v, a.v_bf16, a.at, L, a.H};
  const int tiles = (L + 63) / 64;
  const int Lpad = (L + 127) / 128 * 128;
  float* ksum = a.work;
  float* vmax = ksum + static_cast<int64_t>(tiles) * a.H * 128;
  float* kmean = vmax + static_cast<int64_t>(tiles) * a.H * 128;
  partials_kernel<<<dim3(tiles, a.H), 128, 0, s>>>(ks, vs, ksum, vmax);
  reduce_kernel<<<a.H, 128, 0, s>>>(ksum, vmax, tiles, a.H, L, kmean, a.v_scale);
  quant_kv_kernel<<<dim3(Lpad / 64, a.H), 128, 0, s>>>(ks, vs, kmean, a.v_scale, Lpad, a.k_i8, a.k_scale, a.v_f8);
}

void quant_q_launch(const float* q, int64_t ld_q, int nq, int H, int8_t* q_i8, float* q_scale, cudaStream_t s) {
  const int npad = (nq + 127) / 128 * 128;
  quant_q_kernel<<<dim3(npad / 32, H), 128, 0, s>>>(q, ld_q, nq, npad, q_i8, q_scale);
}

void prep_launch(const PrepArgs& a, cudaStream_t s) {
  prep_kv_launch(a, s);
  quant_q_launch(a.q, a.ld_q, a.nq, a.H, a.q_i8, a.q_scale, s);
}

size_t prep_workspace_floats(int L, int H) {
  const size_t tiles = (static_cast<size_t>(L) + 63) / 64;
  return (2 * tiles + 1) * static_cast<size_t>(H) * 128;
}

}  // namespace sage
}  // namespace wdl
