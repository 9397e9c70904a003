// INT4 group quantization of rows (activations on every call, weights at load) and the unpacking of packed
// weights into the one-code-per-byte layout of the W4A4 GEMM.
//
// Rule (per row, per group of 64 consecutive columns), as w4a4.int4_groups(R, "max") of the reference
// (src/wan_dit_lab/quantization/w4a4.py:86-100) states it for weights and BASELINE's config 1 for activations:
//   scale = max(max|x|, 1e-8) / 7                      fp32, IEEE division
//   code  = clamp(round_half_even(x / scale), -8, 7)   fp32 IEEE division, then rint
// and the stored scale is that fp32 scale rounded to the scale dtype (bf16 in the repo's packs, fp16 in
// BASELINE's config 1), as w4a4.quantize stores it (w4a4.py:174).
//
// One warp per row; a lane holds 8 consecutive columns (16-byte loads of bf16), 8 lanes make one group, so a
// group's max is 3 shuffles. Loads and code stores are 128-bit / 64-bit vector accesses: the kernel is
// HBM-bound (bytes per row: K * in_size + K + K / 64 * 4, plus K / 2 when packing).
#include <type_traits>

#include "common.cuh"
#include "w4a4_quant.h"

namespace wdl {
namespace w4a4 {

__device__ __forceinline__ float round_scale(float s, int scale_dtype) {
  return scale_dtype == 1 ? __half2float(__float2half_rn(s)) : __bfloat162float(__float2bfloat16_rn(s));
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// The byte of a code in the GEMM's operand format: two's complement int8, or the code's value as E4M3 (exact for
// every integer in [-16, 16]).
template <bool kE4M3>
__device__ __forceinline__ uint32_t code_byte(int q) {
  if constexpr (kE4M3)
    return static_cast<uint32_t>(__nv_cvt_float_to_fp8(static_cast<float>(q), __NV_SATFINITE, __NV_E4M3));
  else
    return static_cast<uint32_t>(q) & 0xFFu;
}

// Two codes as float16 halves of a 32-bit word (the folded format's activation operand; exact integers).
__device__ __forceinline__ uint32_t code_pair_f16(int lo, int hi) {
  return static_cast<uint32_t>(__half_as_ushort(__int2half_rn(lo))) |
         (static_cast<uint32_t>(__half_as_ushort(__int2half_rn(hi))) << 16);
}

// kFmt: 0 int8 bytes, 1 E4M3 bytes, 3 float16 (two bytes per code)
template <typename T, bool kSmooth, bool kPack, int kFmt>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ x, int64_t ldx,
                                                            const __nv_bfloat16* __restrict__ smooth, int M, int K,
                                                            int scale_dtype, int8_t* __restrict__ codes,
                                                            float* __restrict__ scales,
                                                            uint8_t* __restrict__ packed) {
  const int lane = threadIdx.x & 31;
  const int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (m >= M) return;
  const T* xr = x + static_cast<int64_t>(m) * ldx;
  // four 256-column chunks per round, their loads issued together (K % 64 == 0: a group of 8 lanes is valid or
  // invalid as a whole)
  for (int k0 = 0; k0 < K; k0 += 1024) {
    float v[4][8];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int k = k0 + c * 256 + lane * 8;
      if (k < K) {
        load8<T>(xr + k, v[c]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (k0 + c * 256 >= K) break;  // uniform over the warp
      const int k = k0 + c * 256 + lane * 8;
      const bool valid = k < K;
      if (kSmooth && valid) {
        float sm[8];
        load8<__nv_bfloat16>(smooth + k, sm);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = __fdiv_rn(v[c][i], sm[i]);
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[c][i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
      if (!valid) continue;
      const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
      const float r = __frcp_rn(scale);
      int q[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = max(-8, min(7, __float2int_rn(div_rn_by(v[c][i], scale, r))));
      if constexpr (kFmt == 3) {
        *reinterpret_cast<uint4*>(codes + (static_cast<int64_t>(m) * K + k) * 2) =
            make_uint4(code_pair_f16(q[0], q[1]), code_pair_f16(q[2], q[3]), code_pair_f16(q[4], q[5]),
                       code_pair_f16(q[6], q[7]));
      } else {
        constexpr bool kE4M3 = kFmt == 1;
        uint2 cw;
        cw.x = code_byte<kE4M3>(q[0]) | (code_byte<kE4M3>(q[1]) << 8) | (code_byte<kE4M3>(q[2]) << 16) |
               (code_byte<kE4M3>(q[3]) << 24);
        cw.y = code_byte<kE4M3>(q[4]) | (code_byte<kE4M3>(q[5]) << 8) | (code_byte<kE4M3>(q[6]) << 16) |
               (code_byte<kE4M3>(q[7]) << 24);
        *reinterpret_cast<uint2*>(codes + static_cast<int64_t>(m) * K + k) = cw;
      }
      if (kPack) {
        uint32_t pw = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) pw |= static_cast<uint32_t>((q[2 * i] & 0xF) | ((q[2 * i + 1] & 0xF) << 4)) << (8 * i);
        *reinterpret_cast<uint32_t*>(packed + static_cast<int64_t>(m) * (K / 2) + k / 2) = pw;
      }
      if ((lane & 7) == 0) scales[static_cast<int64_t>(k / 64) * M + m] = round_scale(scale, scale_dtype);
    }
  }
}

// The prescaled float16 activations (code format 4): the same codes and stored bf16 scales as above, written as
// float16(code * stored scale * 2^-E_m) with one power of two per row, chosen from the row's largest stored scale
// (8 * its largest |code * scale| * 2^-E_m lands in [2^14, 2^15)); rows_scale[m] = 2^E_m. Every value is exact: a
// code has at most 3 significant bits and a bf16 scale 8, and it is a normal float16 number unless its group's
// scale is below 2^-25 of the row's largest (then it rounds to a float16 subnormal, and a value that loses bits is
// reported as kErrInexact in the error word). Two passes over the row
// (the second reads it again from L1 / L2): the scales, then the values.
__device__ __forceinline__ uint32_t exponent_field(float x) { return (__float_as_uint(x) >> 23) & 0xFFu; }

template <typename T, bool kSmooth>
__global__ void __launch_bounds__(256) quantize_rows_pre_kernel(const T* __restrict__ x, int64_t ldx,
                                                                const __nv_bfloat16* __restrict__ smooth, int M,
                                                                int K, uint16_t* __restrict__ out,
                                                                float* __restrict__ rows_scale, uint32_t* err) {
  const int lane = threadIdx.x & 31;
  const int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (m >= M) return;
  const T* xr = x + static_cast<int64_t>(m) * ldx;
  // one chunk of 256 columns per lane round: values, their group's fp32 scale and stored (bf16) scale
  auto group = [&](int k, float (&v)[8], float& scale, float& stored) {
    const bool valid = k < K;
    if (valid) {
      load8<T>(xr + k, v);
      if (kSmooth) {
        float sm[8];
        load8<__nv_bfloat16>(smooth + k, sm);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fdiv_rn(v[i], sm[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
    scale = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
    stored = valid ? __bfloat162float(__float2bfloat16_rn(scale)) : 0.f;
  };
  float top = 0.f;
  for (int k0 = 0; k0 < K; k0 += 256) {
    float v[8], scale, stored;
    group(k0 + lane * 8, v, scale, stored);
    top = fmaxf(top, stored);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
  const uint32_t e = exponent_field(top);  // top in [2^(e-127), 2^(e-126)): 8 top 2^(138-e) in [2^14, 2^15)
  const float down = __uint_as_float((265u - e) << 23);  // 2^(138 - e)
  if (lane == 0) rows_scale[m] = __uint_as_float((e - 11u) << 23);  // 2^(e - 138)
  bool inexact = false;
  for (int k0 = 0; k0 < K; k0 += 256) {
    const int k = k0 + lane * 8;
    float v[8], scale, stored;
    group(k, v, scale, stored);
    if (k >= K) continue;
    const float r = __frcp_rn(scale);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const int q0 = max(-8, min(7, __float2int_rn(div_rn_by(v[i], scale, r))));
      const int q1 = max(-8, min(7, __float2int_rn(div_rn_by(v[i + 1], scale, r))));
      const __half2 h = prescaled_pair(__fmul_rn(static_cast<float>(q0) * stored, down),
                                       __fmul_rn(static_cast<float>(q1) * stored, down), inexact);
      w[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(m) * K + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  report_inexact(inexact, err);
}

// The same values with two warps per row (K <= 512 kChunks): the whole row in registers and one pass over it, so
// that every row of a chunk of tokens is resident at once (as ln_quant_pre_kernel, norm_quant.cu).
template <typename T, bool kSmooth, int kChunks>
__global__ void __launch_bounds__(64, kChunks > 2 ? 8 : 12)
    quantize_rows_pre2_kernel(const T* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ smooth, int M,
                              int K, uint16_t* __restrict__ out, float* __restrict__ rows_scale, uint32_t* err) {
  __shared__ float red[2];
  const int t = threadIdx.x, m = blockIdx.x;
  const T* xr = x + static_cast<int64_t>(m) * ldx;
  float v[kChunks][8];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int k = c * 512 + t * 8;
    if (k < K) {
      load8<T>(xr + k, v[c]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
    }
  }
  float scale[kChunks], stored[kChunks];
  float top = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int k = c * 512 + t * 8;
    const bool valid = k < K;  // uniform over each group of 8 threads
    if (kSmooth && valid) {
      float sm[8];
      load8<__nv_bfloat16>(smooth + k, sm);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = __fdiv_rn(v[c][i], sm[i]);
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[c][i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
    scale[c] = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
    stored[c] = valid ? __bfloat162float(__float2bfloat16_rn(scale[c])) : 0.f;
    top = fmaxf(top, stored[c]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
  if ((t & 31) == 0) red[t >> 5] = top;
  __syncthreads();
  top = fmaxf(red[0], red[1]);
  const uint32_t e = exponent_field(top);
  const float down = __uint_as_float((265u - e) << 23);  // 2^(138 - e)
  if (t == 0) rows_scale[m] = __uint_as_float((e - 11u) << 23);  // 2^(e - 138)
  bool inexact = false;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int k = c * 512 + t * 8;
    if (k >= K) continue;
    const float r = __frcp_rn(scale[c]);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const int q0 = max(-8, min(7, __float2int_rn(div_rn_by(v[c][i], scale[c], r))));
      const int q1 = max(-8, min(7, __float2int_rn(div_rn_by(v[c][i + 1], scale[c], r))));
      const __half2 h = prescaled_pair(__fmul_rn(static_cast<float>(q0) * stored[c], down),
                                       __fmul_rn(static_cast<float>(q1) * stored[c], down), inexact);
      w[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(m) * K + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  report_inexact(inexact, err);
}

// codes [N, K] from qweight [N, K/2]: one thread per 4 packed bytes (8 codes), 32-bit load, 64-bit store.
template <bool kE4M3>
__global__ void unpack_codes_kernel(const uint8_t* __restrict__ qweight, int64_t words, int8_t* __restrict__ codes) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= words) return;
  const uint32_t p = reinterpret_cast<const uint32_t*>(qweight)[i];
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t byte = (p >> (8 * j)) & 0xFFu;
    const int even = static_cast<int>(byte << 28) >> 28;  // sign-extend the low nibble
    const int odd = static_cast<int>((byte >> 4) << 28) >> 28;
    const uint32_t pair = code_byte<kE4M3>(even) | (code_byte<kE4M3>(odd) << 8);
    if (j < 2)
      lo |= pair << (16 * j);
    else
      hi |= pair << (16 * (j - 2));
  }
  reinterpret_cast<uint2*>(codes)[i] = make_uint2(lo, hi);
}

__global__ void scales_to_f32_kernel(const uint16_t* __restrict__ in, int64_t n, int scale_dtype,
                                     float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint16_t b = in[i];
  out[i] = scale_dtype == 1 ? __half2float(__ushort_as_half(b)) : __bfloat162float(__ushort_as_bfloat16(b));
}

template <typename T, int kFmt>
static void launch_rows(const void* x, int64_t ldx, const uint16_t* smooth, int M, int K, int scale_dtype,
                        int8_t* codes, float* scales, uint8_t* packed, cudaStream_t stream) {
  const int threads = 256;
  const int blocks = (M * 32 + threads - 1) / threads;
  const T* xt = static_cast<const T*>(x);
  const __nv_bfloat16* sm = reinterpret_cast<const __nv_bfloat16*>(smooth);
  auto go = [&](auto kernel) {
    kernel<<<blocks, threads, 0, stream>>>(xt, ldx, sm, M, K, scale_dtype, codes, scales, packed);
  };
  if (smooth) {
    if (packed) go(quantize_rows_kernel<T, true, true, kFmt>);
    else go(quantize_rows_kernel<T, true, false, kFmt>);
  } else {
    if (packed) go(quantize_rows_kernel<T, false, true, kFmt>);
    else go(quantize_rows_kernel<T, false, false, kFmt>);
  }
}

void quantize_rows_launch(const void* x, int x_dtype, int64_t ldx, const uint16_t* smooth, int M, int K,
                          int scale_dtype, int code_format, int8_t* codes, float* scales, uint8_t* packed,
                          uint32_t* err, cudaStream_t stream) {
  auto go = [&](auto t) {
    using T = decltype(t);
    if (code_format == 4) {
      const int blocks = (M * 32 + 255) / 256;
      const T* xt = static_cast<const T*>(x);
      const __nv_bfloat16* sm = reinterpret_cast<const __nv_bfloat16*>(smooth);
      uint16_t* out = reinterpret_cast<uint16_t*>(codes);
      if (K <= 4096) {  // two warps per row, the row in registers
        auto go2 = [&](auto chunks) {
          constexpr int C = decltype(chunks)::value;
          if (smooth) quantize_rows_pre2_kernel<T, true, C><<<M, 64, 0, stream>>>(xt, ldx, sm, M, K, out, scales, err);
          else quantize_rows_pre2_kernel<T, false, C><<<M, 64, 0, stream>>>(xt, ldx, sm, M, K, out, scales, err);
        };
        const int chunks = (K + 511) / 512;
        if (chunks <= 2) go2(std::integral_constant<int, 2>{});
        else if (chunks <= 4) go2(std::integral_constant<int, 4>{});
        else if (chunks <= 6) go2(std::integral_constant<int, 6>{});
        else go2(std::integral_constant<int, 8>{});
        return;
      }
      if (smooth) quantize_rows_pre_kernel<T, true><<<blocks, 256, 0, stream>>>(xt, ldx, sm, M, K, out, scales, err);
      else quantize_rows_pre_kernel<T, false><<<blocks, 256, 0, stream>>>(xt, ldx, sm, M, K, out, scales, err);
      return;
    }
    if (code_format == 3) launch_rows<T, 3>(x, ldx, smooth, M, K, scale_dtype, codes, scales, packed, stream);
    else if (code_format != 0) launch_rows<T, 1>(x, ldx, smooth, M, K, scale_dtype, codes, scales, packed, stream);
    else launch_rows<T, 0>(x, ldx, smooth, M, K, scale_dtype, codes, scales, packed, stream);
  };
  if (x_dtype == 2) go(float{});
  else go(__nv_bfloat16{});
}

void unpack_weight_launch(const uint8_t* qweight, const uint16_t* wscales, int scale_dtype, int N, int K,
                          int code_format, int8_t* codes, float* scales, cudaStream_t stream) {
  const int64_t words = static_cast<int64_t>(N) * K / 8;
  const unsigned grid = static_cast<unsigned>((words + 255) / 256);
  if (code_format != 0)
    unpack_codes_kernel<true><<<grid, 256, 0, stream>>>(qweight, words, codes);
  else
    unpack_codes_kernel<false><<<grid, 256, 0, stream>>>(qweight, words, codes);
  const int64_t ns = static_cast<int64_t>(K / 64) * N;
  scales_to_f32_kernel<<<static_cast<unsigned>((ns + 255) / 256), 256, 0, stream>>>(wscales, ns, scale_dtype, scales);
}

}  // namespace w4a4
}  // namespace wdl
