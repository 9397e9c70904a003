// 3D RoPE, the FP8 (E4M3) KV-cache store, and the fused QK preparation of a Wan block's self-attention.
//
//  * store_kv_fp8 — the reference's kernels/cache_fp8.py:23-105 and KVCache.store (generation/causal.py:177-184)
//    whose arithmetic is quantization/fp8.py:37-41 quantize_rows: per row (token, head) of D channels,
//    scale = max(max|x|, 1e-12) / 448, e4m3 = round-to-nearest-even(x / scale), written into
//    cache[b, at + t, h, :] and its scale into scales[b, at + t, h]. One warp per row.
//  * rope_apply — kernels/rope_triton.py:15-64 / models/rope.py:12-31: token t of the grid (f, h, w) of its
//    sample has positions (start + t / (h w), t / w % h, t % w); pair i of D/2 rotates by the angle of the time,
//    height or width axis (pairs split D/2 - 2 (D/2/3), D/2/3, D/2/3); x1' = x1 c - x2 s, x2' = x2 c + x1 s,
//    products and difference rounded separately (no FMA), in float32, or float64 when the input or the table
//    is float64; tokens past f h w are copied. One thread per pair.
//  * qkv_prep — the chain of FusedQKVAttention.forward (quantization/w4a4.py:252-262) on one QKV row:
//    RMSNorm over all heads of q and of k (models/rms_norm.py:10-13: float32 statistics, rounded to bf16,
//    times the float32 weight), RoPE of both (float32 table), then K and V stored into the FP8 cache at
//    `at`, Q and K written in float32 for the attention, all from one read of the row. One CTA per token.
#include "common.cuh"
#include "rope_kv.h"

namespace wdl {
namespace ropekv {

__device__ __forceinline__ uint8_t e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

template <typename T>
__device__ __forceinline__ float load_as_float(const T* p);
template <>
__device__ __forceinline__ float load_as_float<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_as_float<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float load_as_float<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float load_as_float<double>(const double* p) { return static_cast<float>(*p); }

// ------------------------------------------------------------------------------------------------------------
// store_kv_fp8: warp per (b, t, h) row; lanes stride over D.
template <typename T>
__device__ void store_row(const T* __restrict__ x, const int64_t* st, int b, int t, int h, int D,
                          uint8_t* __restrict__ cache, float* __restrict__ scales, int64_t row_out) {
  const int lane = threadIdx.x & 31;
  const T* base = x + b * st[0] + t * st[1] + h * st[2];
  float amax = 0.f;
  for (int d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(load_as_float<T>(base + d * st[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const float scale = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  uint8_t* out = cache + row_out * D;
  for (int d = lane; d < D; d += 32) out[d] = e4m3(__fdiv_rn(load_as_float<T>(base + d * st[3]), scale));
  if (lane == 0) scales[row_out] = scale;
}

template <typename TK, typename TV>
__global__ void store_kv_kernel(const TK* __restrict__ k, const TV* __restrict__ v, StoreArgs a) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t rows = static_cast<int64_t>(a.B) * a.N * a.H;
  if (row >= rows) return;
  const int h = static_cast<int>(row % a.H), t = static_cast<int>(row / a.H % a.N), b = static_cast<int>(row / (static_cast<int64_t>(a.H) * a.N));
  const int64_t out_row = (static_cast<int64_t>(b) * a.capacity + a.at + t) * a.H + h;
  if (blockIdx.y == 0)
    store_row<TK>(k, a.k_strides, b, t, h, a.D, a.cache_k, a.cache_ks, out_row);
  else
    store_row<TV>(v, a.v_strides, b, t, h, a.D, a.cache_v, a.cache_vs, out_row);
}

template <typename TK>
static void launch_store_v(const StoreArgs& a, int v_dtype, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(a.B) * a.N * a.H;
  const dim3 grid(static_cast<unsigned>((rows * 32 + 255) / 256), 2);
  const TK* k = static_cast<const TK*>(a.k);
  if (v_dtype == 2) store_kv_kernel<TK, float><<<grid, 256, 0, s>>>(k, static_cast<const float*>(a.v), a);
  else if (v_dtype == 1) store_kv_kernel<TK, __half><<<grid, 256, 0, s>>>(k, static_cast<const __half*>(a.v), a);
  else store_kv_kernel<TK, __nv_bfloat16><<<grid, 256, 0, s>>>(k, static_cast<const __nv_bfloat16*>(a.v), a);
}

void store_kv_launch(const StoreArgs& a, cudaStream_t s) {
  if (a.k_dtype == 2) launch_store_v<float>(a, a.v_dtype, s);
  else if (a.k_dtype == 1) launch_store_v<__half>(a, a.v_dtype, s);
  else launch_store_v<__nv_bfloat16>(a, a.v_dtype, s);
}

// ------------------------------------------------------------------------------------------------------------
// rope_apply: thread per (b, t, h, pair).
template <typename TC>
__device__ __forceinline__ TC mul_rn(TC a, TC b);
template <>
__device__ __forceinline__ float mul_rn<float>(float a, float b) { return __fmul_rn(a, b); }
template <>
__device__ __forceinline__ double mul_rn<double>(double a, double b) { return __dmul_rn(a, b); }
template <typename TC>
__device__ __forceinline__ TC add_rn(TC a, TC b);
template <>
__device__ __forceinline__ float add_rn<float>(float a, float b) { return __fadd_rn(a, b); }
template <>
__device__ __forceinline__ double add_rn<double>(double a, double b) { return __dadd_rn(a, b); }

template <typename T>
__device__ __forceinline__ double load_as_double(const T* p) {
  if constexpr (std::is_same<T, double>::value) return *p;
  else return static_cast<double>(load_as_float<T>(p));
}

template <typename TO, typename TC>
__device__ __forceinline__ TO store_cast(TC v) {
  if constexpr (std::is_same<TO, double>::value) return static_cast<double>(v);
  else if constexpr (std::is_same<TO, float>::value) return static_cast<float>(v);
  else if constexpr (std::is_same<TO, __half>::value) return __float2half_rn(static_cast<float>(v));
  else return __float2bfloat16_rn(static_cast<float>(v));  // float64 -> bf16 through float32, as PyTorch casts
}

template <typename TX, typename TF, typename TO, typename TC>
__global__ void rope_kernel(const TX* __restrict__ x, const TF* __restrict__ freq, TO* __restrict__ out, RopeArgs a) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int pairs = a.D / 2;
  const int64_t total = static_cast<int64_t>(a.B) * a.L * a.H * pairs;
  if (i >= total) return;
  const int pair = static_cast<int>(i % pairs);
  const int h = static_cast<int>(i / pairs % a.H);
  const int t = static_cast<int>(i / (static_cast<int64_t>(pairs) * a.H) % a.L);
  const int b = static_cast<int>(i / (static_cast<int64_t>(pairs) * a.H * a.L));
  const int gf = a.grids[3 * b], gh = a.grids[3 * b + 1], gw = a.grids[3 * b + 2];
  const int spatial = pairs / 3, time_pairs = pairs - 2 * spatial;
  const TX* px = x + b * a.x_strides[0] + t * a.x_strides[1] + h * a.x_strides[2] + (2 * pair) * a.x_strides[3];
  TC even, odd;
  if constexpr (std::is_same<TC, double>::value) {
    even = load_as_double<TX>(px);
    odd = load_as_double<TX>(px + a.x_strides[3]);
  } else {
    even = load_as_float<TX>(px);
    odd = load_as_float<TX>(px + a.x_strides[3]);
  }
  TO* po = out + ((static_cast<int64_t>(b) * a.L + t) * a.H + h) * a.D + 2 * pair;
  if (t < gf * gh * gw) {
    const int pos = pair < time_pairs ? a.start + t / (gh * gw) : (pair < time_pairs + spatial ? t / gw % gh : t % gw);
    const TF* pc = freq + pos * a.f_strides[1] + pair * a.f_strides[2];
    TC c, s;
    if constexpr (std::is_same<TC, double>::value) {
      c = load_as_double<TF>(pc);
      s = load_as_double<TF>(pc + a.f_strides[0]);
    } else {
      c = load_as_float<TF>(pc);
      s = load_as_float<TF>(pc + a.f_strides[0]);
    }
    po[0] = store_cast<TO, TC>(add_rn<TC>(mul_rn<TC>(even, c), -mul_rn<TC>(odd, s)));
    po[1] = store_cast<TO, TC>(add_rn<TC>(mul_rn<TC>(odd, c), mul_rn<TC>(even, s)));
  } else {  // padding: copied verbatim
    po[0] = store_cast<TO, TC>(even);
    po[1] = store_cast<TO, TC>(odd);
  }
}

template <typename TX, typename TF, typename TO>
static void rope_dispatch_c(const RopeArgs& a, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(a.B) * a.L * a.H * (a.D / 2);
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  const bool f64 = std::is_same<TX, double>::value || std::is_same<TF, double>::value;
  if (f64)
    rope_kernel<TX, TF, TO, double><<<grid, 256, 0, s>>>(static_cast<const TX*>(a.x), static_cast<const TF*>(a.freq),
                                                         static_cast<TO*>(a.out), a);
  else
    rope_kernel<TX, TF, TO, float><<<grid, 256, 0, s>>>(static_cast<const TX*>(a.x), static_cast<const TF*>(a.freq),
                                                        static_cast<TO*>(a.out), a);
}

template <typename TX, typename TF>
static void rope_dispatch_o(const RopeArgs& a, cudaStream_t s) {
  switch (a.out_dtype) {
    case 0: rope_dispatch_c<TX, TF, __nv_bfloat16>(a, s); break;
    case 1: rope_dispatch_c<TX, TF, __half>(a, s); break;
    case 2: rope_dispatch_c<TX, TF, float>(a, s); break;
    default: rope_dispatch_c<TX, TF, double>(a, s); break;
  }
}

template <typename TX>
static void rope_dispatch_f(const RopeArgs& a, cudaStream_t s) {
  if (a.freq_dtype == 3) rope_dispatch_o<TX, double>(a, s);
  else rope_dispatch_o<TX, float>(a, s);
}

void rope_launch(const RopeArgs& a, cudaStream_t s) {
  switch (a.x_dtype) {
    case 0: rope_dispatch_f<__nv_bfloat16>(a, s); break;
    case 1: rope_dispatch_f<__half>(a, s); break;
    case 2: rope_dispatch_f<float>(a, s); break;
    default: rope_dispatch_f<double>(a, s); break;
  }
}

// ------------------------------------------------------------------------------------------------------------
// qkv_prep: one CTA of kThreads threads per token. Row layout: q | k | v, each H * 128 bf16 (dim = H * 128).
// Thread t holds 8 consecutive channels of each (kThreads * 8)-channel pass; 16 lanes cover one head of 128
// channels. dim <= 3072 runs 384 threads, one pass: a thread's dependent chain of loads, reductions and stores
// bounds these rows (128 threads and three passes measured slower).
template <int kWarps>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// 8 values / scale rounded to E4M3 (the division correctly rounded, Markstein's method), packed in 8 bytes.
__device__ __forceinline__ uint2 e4m3x8(const float (&y)[8], float scale) {
  const float r = __frcp_rn(scale);
  uint32_t w[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i / 4] |= static_cast<uint32_t>(e4m3(div_rn_by(y[i], scale, r))) << (8 * (i % 4));
  return make_uint2(w[0], w[1]);
}

template <int kThreads, int kPasses>
__global__ void __launch_bounds__(kThreads) qkv_prep_kernel(QkvPrepArgs a) {
  constexpr int kStride = kThreads * 8;
  __shared__ float red[kThreads / 32];
  const int t = blockIdx.x;  // token of the chunk
  const int tid = threadIdx.x;
  const int dim = a.dim;  // this call's channels of q (a multiple of 128, at most kPasses * kStride)
  const __nv_bfloat16* row = a.qkv + static_cast<int64_t>(t) * a.ld_qkv;
  const int gh = a.grid_h, gw = a.grid_w;
  const int pos_t = a.start + t / (gh * gw), pos_h = t / gw % gh, pos_w = t % gw;
  const int time_pairs = 64 - 2 * 21;  // head_dim 128: 22 time pairs, 21 height, 21 width

  // q (part 0) and k (part 1): RMSNorm over the whole row of norm_dim channels, RoPE per head. A thread whose
  // channels lie past dim (a partial last pass) joins every shuffle and sum but loads and stores nothing; the
  // 16 lanes of a head are all in or all out.
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    float v[kPasses][8];
    float ss = 0.f;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int c0 = p * kStride + tid * 8;
      if (c0 < dim) {
        load8_bf16(row + part * dim + c0, v[p]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[p][i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[p][i], v[p][i], ss);
    }
    const float own = block_sum<kThreads / 32>(ss, red);
    const float total = a.sumsq ? __ldg(a.sumsq + static_cast<int64_t>(t) * 2 + part) : own;
    const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(a.norm_dim)), a.eps));
    const float* w = part == 0 ? a.norm_q : a.norm_k;
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int c0 = p * kStride + tid * 8;  // channel of v[p][0]
      const bool act = c0 < dim;
      const int head = c0 >> 7, d0 = c0 & 127;
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // (x * rsqrt(mean + eps)) rounded to x's bf16, then times the float32 weight
        const float n = __bfloat162float(__float2bfloat16_rn(__fmul_rn(v[p][i], r)));
        y[i] = act ? __fmul_rn(n, __ldg(w + c0 + i)) : 0.f;
      }
      // RoPE on the 4 pairs (float32 table; products and difference rounded separately)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pair = (d0 >> 1) + j;
        const int pos = pair < time_pairs ? pos_t : (pair < time_pairs + 21 ? pos_h : pos_w);
        const float c = __ldg(a.freq + pos * a.freq_positions_stride + pair);
        const float s = __ldg(a.freq + a.freq_table_stride + pos * a.freq_positions_stride + pair);
        const float e = y[2 * j], o = y[2 * j + 1];
        y[2 * j] = __fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s));
        y[2 * j + 1] = __fadd_rn(__fmul_rn(o, c), __fmul_rn(e, s));
      }
      if (act) {
        float* dst = (part == 0 ? a.q_out : a.k_out) + static_cast<int64_t>(t) * dim + c0;
        *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
      }
      if (part == 1 && a.cache_k) {  // FP8 store of the rotated key row of this head (16 lanes)
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[i]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        if (act) {
          const float scale = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
          const int64_t crow = static_cast<int64_t>(a.at + t) * (dim / 128) + head;
          const uint2 q8 = e4m3x8(y, scale);
          *reinterpret_cast<uint2*>(a.cache_k + crow * 128 + d0) = q8;
          if ((tid & 15) == 0) a.cache_ks[crow] = scale;
        }
      }
    }
  }
  // v (part 2): FP8 store of each head row
  if (a.cache_v) {
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int c0 = p * kStride + tid * 8;
      const bool act = c0 < dim;
      const int head = c0 >> 7, d0 = c0 & 127;
      float y[8];
      if (act) {
        load8_bf16(row + 2 * dim + c0, y);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = 0.f;
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
      if (act) {
        const float scale = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
        const int64_t crow = static_cast<int64_t>(a.at + t) * (dim / 128) + head;
        const uint2 q8 = e4m3x8(y, scale);
        *reinterpret_cast<uint2*>(a.cache_v + crow * 128 + d0) = q8;
        if ((tid & 15) == 0) a.cache_vs[crow] = scale;
      }
    }
  }
}

void qkv_prep_launch(const QkvPrepArgs& a, cudaStream_t s) {
  if (a.dim <= 3072) {
    qkv_prep_kernel<384, 1><<<a.n, 384, 0, s>>>(a);
    return;
  }
  qkv_prep_kernel<128, 4><<<a.n, 128, 0, s>>>(a);
}

}  // namespace ropekv
}  // namespace wdl
