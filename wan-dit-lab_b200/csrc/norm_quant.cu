// The normalizations of a Wan block fused with what consumes them:
//
//  * ln_quant — LayerNorm over dim channels (models/layer_norm.py:5-7: float32 statistics, eps 1e-6, optional
//    affine weight / bias as norm3), its result rounded to the residual stream's dtype when that is bf16
//    (.type_as(X)), the AdaLN modulation y * (1 + scale) + shift with scale / shift rows of
//    (time_in + modulation) (models/block.py:75-79, each product and sum rounded in float32), the cast to bf16
//    of the linear layer that follows (PackedW4A4Linear.forward, quantization/w4a4.py:229-231), then that
//    layer's activation quantization: division by its smoothing vector and symmetric INT4 groups of 64
//    (scale = max(max|x|, 1e-8) / 7, round half to even, codes in the GEMM's operand format). One CTA of 128 threads per row.
//  * rms_rows — RMSNorm of rows (models/rms_norm.py:10-13): x * rsqrt(mean(x^2) + eps) rounded to bf16, times
//    the float32 weight; the query norm of cross-attention (models/multi_head_attention.py:118).
//  * modulation — (time_in + modulation) of every block at once (models/block.py:75): [blocks, 6, dim] fp32.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "norm_quant.h"

namespace wdl {
namespace norm {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x, v[2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One CTA of 128 threads per row: thread t holds channels c * 1024 + 8 t .. + 7 of every 1024-channel chunk c
// (the last chunk may be partial: K % 256 == 0, so a group of 64 channels is wholly present or absent), so 8
// consecutive threads hold one group of 64 (its max: 3 shuffles) and the row statistics are two CTA sums.
constexpr int kRowThreads = 128;
constexpr int kRowChunks = 4;  // K <= 4096

__device__ __forceinline__ float block_sum128(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}

// The CTA's sum (kWarps warps), its warps' sums added pairwise in a fixed order.
template <int kWarps>
__device__ __forceinline__ float block_sum(float v, float* red) {
  if constexpr (kWarps == 4) {
    return block_sum128(v, red);
  } else {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float p[kWarps];
#pragma unroll
    for (int i = 0; i < kWarps; ++i) p[i] = red[i];
#pragma unroll
    for (int w = 1; w < kWarps; w *= 2)
#pragma unroll
      for (int i = 0; i + w < kWarps; i += 2 * w) p[i] += p[i + w];
    return p[0];
  }
}

__device__ __forceinline__ uint32_t code_byte(int q, int fmt) {
  return fmt != 0 ? static_cast<uint32_t>(__nv_cvt_float_to_fp8(static_cast<float>(q), __NV_SATFINITE, __NV_E4M3))
                  : (static_cast<uint32_t>(q) & 0xFFu);
}

// kKeep: also write the bf16 layer input to a.x_out. kPre: code format 4, the prescaled float16 activations
// float16(code * stored scale * 2^-E_m) with the row's 2^E_m in a.scales[m] (E_m from the row's largest stored
// scale, as quantize_rows_pre_kernel: w4a4_quant.cu); the codes and scales are those of the other formats.
// kThreads threads per row, kChunks chunks of kThreads * 8 channels (kThreads * 8 * kChunks >= K). The prescaled
// format with K <= 3072 runs 384 threads, one chunk each: a thread's dependent chain of loads and arithmetic is
// what bounds these rows, and one chunk a thread shortens it threefold.
template <typename TX, bool kKeep, bool kPre, int kThreads = kRowThreads, int kChunks = kRowChunks>
__global__ void __launch_bounds__(kThreads, kThreads == 128 ? (kPre ? 4 : 6) : 3)
    ln_quant_kernel(const TX* __restrict__ x, LnQuantArgs a) {
  constexpr int kWarps = kThreads / 32, kStride = kThreads * 8;
  __shared__ float red[kWarps];
  const int t = threadIdx.x, m = blockIdx.x;
  const int K = a.K;
  const TX* row = x + static_cast<int64_t>(m) * a.ldx;
  float v[kChunks][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int k = c * kStride + t * 8;
    if (k < K) {
      load8<TX>(row + k, v[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[c][i];
    }
  }
  const float mean = __fdiv_rn(block_sum<kWarps>(s, red), static_cast<float>(K));
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c)
    if (c * kStride + t * 8 < K)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[c][i] - mean;
        ss = fmaf(d, d, ss);
      }
  const float rstd = __frsqrt_rn(__fadd_rn(__fdiv_rn(block_sum<kWarps>(ss, red), static_cast<float>(K)), a.eps));
  uint8_t* codes = a.codes + static_cast<int64_t>(m) * K;
  float pre_scale[kChunks], pre_stored[kChunks];  // kPre: each chunk's group scale and stored scale
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    if (c * kStride >= K) break;  // uniform over the CTA
    const int k = c * kStride + t * 8;
    const bool valid = k < K;  // uniform over each group of 8 threads
    float y[8];
    if (valid) {
      float w[8], b[8], sh[8], sc[8], sm[8], xb[8];
      if (a.ln_w) {
        load8<float>(a.ln_w + k, w);
        load8<float>(a.ln_b + k, b);
      }
      if (a.mod_shift) {
        load8<float>(a.mod_shift + k, sh);
        load8<float>(a.mod_scale + k, sc);
      }
      if (a.smooth) load8<__nv_bfloat16>(a.smooth + k, sm);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float u = __fmul_rn(v[c][i] - mean, rstd);
        if (a.ln_w) u = __fadd_rn(__fmul_rn(u, w[i]), b[i]);
        if (a.round_ln_bf16) u = bf16r(u);
        if (a.mod_shift) u = __fadd_rn(__fmul_rn(u, __fadd_rn(1.f, sc[i])), sh[i]);
        u = bf16r(u);  // the linear layer's input is bf16
        if constexpr (kKeep) xb[i] = u;
        if (a.smooth) u = __fdiv_rn(u, sm[i]);
        y[i] = u;
      }
      if constexpr (kKeep) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat162 p2 = __floats2bfloat162_rn(xb[2 * i], xb[2 * i + 1]);
          pk[i] = *reinterpret_cast<const uint32_t*>(&p2);
        }
        *reinterpret_cast<uint4*>(a.x_out + static_cast<int64_t>(m) * a.ld_xo + k) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
    if constexpr (kPre) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = y[i];  // kept for the second pass
      pre_scale[c] = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
      pre_stored[c] = valid ? bf16r(pre_scale[c]) : 0.f;
      continue;
    }
    if (!valid) continue;
    const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
    const float r = __frcp_rn(scale);
    if (a.code_format == 3) {  // float16 codes, two bytes each
      uint32_t hw[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const int q0 = max(-8, min(7, __float2int_rn(div_rn_by(y[i], scale, r))));
        const int q1 = max(-8, min(7, __float2int_rn(div_rn_by(y[i + 1], scale, r))));
        hw[i / 2] = static_cast<uint32_t>(__half_as_ushort(__int2half_rn(q0))) |
                    (static_cast<uint32_t>(__half_as_ushort(__int2half_rn(q1))) << 16);
      }
      *reinterpret_cast<uint4*>(a.codes + (static_cast<int64_t>(m) * K + k) * 2) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    } else {
      uint32_t wd[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = max(-8, min(7, __float2int_rn(div_rn_by(y[i], scale, r))));
        wd[i / 4] |= code_byte(q, a.code_format) << (8 * (i % 4));
      }
      *reinterpret_cast<uint2*>(codes + k) = make_uint2(wd[0], wd[1]);
    }
    if ((t & 7) == 0) {
      const float stored = a.scale_dtype == 1 ? __half2float(__float2half_rn(scale)) : bf16r(scale);
      const int64_t i = static_cast<int64_t>(k / 64) * a.M + m;
      a.scales[i] = stored;
    }
  }
  if constexpr (kPre) {
    float top = 0.f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c)
      if (c * kStride < K) top = fmaxf(top, pre_stored[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
    __syncthreads();
    if ((t & 31) == 0) red[t >> 5] = top;
    __syncthreads();
    top = red[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) top = fmaxf(top, red[i]);
    const uint32_t e = (__float_as_uint(top) >> 23) & 0xFFu;  // 8 top 2^(138-e) in [2^14, 2^15)
    const float down = __uint_as_float((265u - e) << 23);
    if (t == 0) a.scales[m] = __uint_as_float((e - 11u) << 23);  // 2^(e - 138)
    uint16_t* out = reinterpret_cast<uint16_t*>(a.codes) + static_cast<int64_t>(m) * K;
    bool inexact = false;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int k = c * kStride + t * 8;
      if (k >= K) continue;
      const float scale = pre_scale[c], stored = pre_stored[c];
      const float r = __frcp_rn(scale);
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const int q0 = max(-8, min(7, __float2int_rn(div_rn_by(v[c][i], scale, r))));
        const int q1 = max(-8, min(7, __float2int_rn(div_rn_by(v[c][i + 1], scale, r))));
        const __half2 h = prescaled_pair(__fmul_rn(static_cast<float>(q0) * stored, down),
                                         __fmul_rn(static_cast<float>(q1) * stored, down), inexact);
        w[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(out + k) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    report_inexact(inexact, a.err);
  }
}

void ln_quant_launch(const LnQuantArgs& a, cudaStream_t s) {
  if (a.M == 0) return;
  auto go = [&](auto xt, auto keep, auto pre) {
    using TX = decltype(xt);
    ln_quant_kernel<TX, decltype(keep)::value, decltype(pre)::value>
        <<<a.M, kRowThreads, 0, s>>>(static_cast<const TX*>(a.x), a);
  };
  using T_ = std::true_type;
  using F_ = std::false_type;
  const bool pre = a.code_format == 4, keep = a.x_out != nullptr;
  if (pre && a.K <= 3072) {  // 384 threads a row, one chunk each
    auto go384 = [&](auto xt, auto kp) {
      using TX = decltype(xt);
      ln_quant_kernel<TX, decltype(kp)::value, true, 384, 1><<<a.M, 384, 0, s>>>(static_cast<const TX*>(a.x), a);
    };
    if (a.x_f32) keep ? go384(float{}, T_{}) : go384(float{}, F_{});
    else keep ? go384(__nv_bfloat16{}, T_{}) : go384(__nv_bfloat16{}, F_{});
    return;
  }
  if (a.x_f32) {
    if (pre) keep ? go(float{}, T_{}, T_{}) : go(float{}, F_{}, T_{});
    else keep ? go(float{}, T_{}, F_{}) : go(float{}, F_{}, F_{});
  } else {
    const __nv_bfloat16 b{};
    if (pre) keep ? go(b, T_{}, T_{}) : go(b, F_{}, T_{});
    else keep ? go(b, T_{}, F_{}) : go(b, F_{}, F_{});
  }
}

// Same thread layout as ln_quant: one CTA of 128 threads per row.
// sumsq (nullable): the sum of squares of each row over all norm_dim channels, when this call holds only a slice
// of them (a tensor-parallel shard: the slices' sums added across shards); else the row's own sum over K = norm_dim.
// kThreads threads a row, kChunks chunks of kThreads * 8 channels; K <= 3072 runs 384 threads, one chunk each.
template <int kThreads = kRowThreads, int kChunks = kRowChunks>
__global__ void __launch_bounds__(kThreads, kThreads == kRowThreads ? 8 : 4)
    rms_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int K, const float* __restrict__ w, float eps,
                    const float* __restrict__ sumsq, int norm_dim, float* __restrict__ out, int64_t ldo) {
  constexpr int kStride = kThreads * 8;
  __shared__ float red[kThreads / 32];
  const int t = threadIdx.x, m = blockIdx.x;
  const __nv_bfloat16* row = x + static_cast<int64_t>(m) * ldx;
  float v[kChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int k = c * kStride + t * 8;
    if (k < K) {
      load8<__nv_bfloat16>(row + k, v[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
    }
  }
  const float total = block_sum<kThreads / 32>(ss, red);
  const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(sumsq ? __ldg(sumsq + m) : total, static_cast<float>(norm_dim)), eps));
  float* o = out + static_cast<int64_t>(m) * ldo;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int k = c * kStride + t * 8;
    if (k < K) {
      float wk[8], y[8];
      load8<float>(w + k, wk);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = __fmul_rn(bf16r(__fmul_rn(v[c][i], r)), wk[i]);
      *reinterpret_cast<float4*>(o + k) = make_float4(y[0], y[1], y[2], y[3]);
      *reinterpret_cast<float4*>(o + k + 4) = make_float4(y[4], y[5], y[6], y[7]);
    }
  }
}

void rms_rows_launch(const __nv_bfloat16* x, int64_t ldx, int M, int K, const float* w, float eps, const float* sumsq,
                     int norm_dim, float* out, int64_t ldo, cudaStream_t s) {
  if (M == 0) return;
  if (K <= 3072) rms_rows_kernel<384, 1><<<M, 384, 0, s>>>(x, ldx, K, w, eps, sumsq, norm_dim, out, ldo);
  else rms_rows_kernel<><<<M, kRowThreads, 0, s>>>(x, ldx, K, w, eps, sumsq, norm_dim, out, ldo);
}

// Sums of squares of `parts` slices of K channels of each bf16 row (slice p starts at channel p * part_stride):
// out[m * parts + p]. Same thread layout and summation order as rms_rows. A tensor-parallel shard's share of an
// RMSNorm over channels split across shards (the q / k norms of self-attention, the query norm of cross-attention).
__global__ void __launch_bounds__(kRowThreads, 8) rows_sumsq_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                 int K, int parts, int64_t part_stride,
                                                                 float* __restrict__ out) {
  __shared__ float red[kRowThreads / 32];
  const int t = threadIdx.x, m = blockIdx.x;
  for (int p = 0; p < parts; ++p) {
    const __nv_bfloat16* row = x + static_cast<int64_t>(m) * ldx + p * part_stride;
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
      const int k = c * 1024 + t * 8;
      if (k < K) {
        float v[8];
        load8<__nv_bfloat16>(row + k, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
      }
    }
    const float total = block_sum128(ss, red);
    if (t == 0) out[static_cast<int64_t>(m) * parts + p] = total;
  }
}

void rows_sumsq_launch(const __nv_bfloat16* x, int64_t ldx, int M, int K, int parts, int64_t part_stride, float* out,
                       cudaStream_t s) {
  if (M == 0) return;
  rows_sumsq_kernel<<<M, kRowThreads, 0, s>>>(x, ldx, K, parts, part_stride, out);
}

// The residual update after a row-parallel layer's shards have been summed (tensor-parallel blocks): x += gate *
// float(bf16(partial + bias)) (gate 1 when null), the arithmetic of the GEMM's residual epilogue. Four columns per
// thread (N % 4 == 0, 16-byte aligned rows).
__global__ void residual_update_kernel(const float* __restrict__ partial, int64_t ldp, const float* __restrict__ bias,
                                       const float* __restrict__ gate, float* __restrict__ x, int64_t ldx, int M,
                                       int N) {
  const int64_t quads = static_cast<int64_t>(M) * (N / 4);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < quads;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / (N / 4)), n = static_cast<int>(i % (N / 4)) * 4;
    const float4 p = *reinterpret_cast<const float4*>(partial + static_cast<int64_t>(m) * ldp + n);
    float4* xp = reinterpret_cast<float4*>(x + static_cast<int64_t>(m) * ldx + n);
    const float4 xv = *xp;
    const float pv[4] = {p.x, p.y, p.z, p.w};
    float v[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float o = bf16r(pv[j] + (bias ? __ldg(bias + n + j) : 0.f));
      v[j] = gate ? __fadd_rn(v[j], __fmul_rn(o, __ldg(gate + n + j))) : __fadd_rn(v[j], o);
    }
    *xp = make_float4(v[0], v[1], v[2], v[3]);
  }
}

void residual_update_launch(const float* partial, int64_t ldp, const float* bias, const float* gate, float* x,
                            int64_t ldx, int M, int N, cudaStream_t s) {
  const int64_t quads = static_cast<int64_t>(M) * (N / 4);
  if (quads == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((quads + 255) / 256, 148 * 8));
  residual_update_kernel<<<blocks, 256, 0, s>>>(partial, ldp, bias, gate, x, ldx, M, N);
}

__global__ void modulation_kernel(const float* __restrict__ time_in, const float* __restrict__ modulation, int64_t n,
                                  int64_t per_block, float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __fadd_rn(time_in[i % per_block], modulation[i]);
}

void modulation_launch(const float* time_in, const float* modulation, int blocks, int dim, float* out, cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(blocks) * 6 * dim;
  modulation_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(time_in, modulation, n, 6 * dim, out);
}

}  // namespace norm
}  // namespace wdl
