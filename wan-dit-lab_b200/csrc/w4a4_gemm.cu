// W4A4 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8), with the per-group scale promotion of
// SVDQuant's INT4 linear:
//
//   y[m, n] = sum_g  sx[g, m] * sw[g, n] * P_g[m, n],     P_g[m, n] = sum_{k in group g} xq[m, k] * wq[n, k]
//
// xq, wq are 4-bit integers held one per byte (int8 in [-8, 7], or [0, 15] for the unsigned hidden layer of
// the fused MLP), groups are 64 consecutive k. P_g is exact in 32-bit integers: the tensor core accumulates
// each group into its own TMEM buffer; epilogue warps read it (tcgen05.ld), convert, scale by
// sx[g, m] * sw[g, n] and add it to fp32 accumulators in registers. This is the arithmetic of Nunchaku's
// gemm_w4a4 (called from the reference's native/ops/w4a4_ops.cpp:36), whose int4 mma.sync tiles accumulate a
// group in int32 registers and promote it the same way.
//
// Tile 128 x 256 x 128 (two groups per pipeline stage), one CTA per SM, 12 warps:
//   warp 0      TMA producer: A, B tiles (128-byte swizzle) and the weight scales of the stage
//   warp 1      TMEM owner and MMA issuer: 2 x K=32 MMAs per group into TMEM buffer (group % 2)
//   warps 4-11  promotion + epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and columns
//               128 ((w - 4) / 4) .. +127, keeps 128 fp32 accumulators per thread
// TMEM: 2 buffers x 256 columns of int32 = all 512 columns.
#include "common.cuh"
#include "w4a4_gemm.h"

namespace wdl {
namespace w4a4 {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4, GROUP = 64;
constexpr int GPS = BK / GROUP;  // groups per stage
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, WS_BYTES = GPS * BN * 4;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) Smem {
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  float ws[STAGES][GPS][BN];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t ws_empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + alignment slack of the dynamic buffer

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

__device__ __forceinline__ float4 lds128(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ float partial(uint32_t p, bool fp8) {
  return fp8 ? __uint_as_float(p) : static_cast<float>(static_cast<int32_t>(p));
}

// acc += P * (sx * w) for two adjacent columns. P is the group partial as the tensor core left it: fp32 bits
// (E4M3-coded operands) or int32 (int8 codes). kPacked: one f32x2 multiply and one f32x2 fused multiply-add
// for the pair; else two scalar multiplies and two scalar FMAs (same roundings either way).
template <bool kFp8, bool kPacked>
__device__ __forceinline__ void promote2(uint64_t& acc, uint32_t p0, uint32_t p1, float w0, float w1, uint64_t sx2) {
  if constexpr (kPacked) {
    uint64_t p;
    if constexpr (kFp8) {
      asm("mov.b64 %0, {%1, %2};" : "=l"(p) : "r"(p0), "r"(p1));
    } else {
      p = pack2(partial(p0, false), partial(p1, false));
    }
    uint64_t sc;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(sc) : "l"(sx2), "l"(pack2(w0, w1)));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(p), "l"(sc));
  } else {
    const float sx = unpack2(sx2).x;
    float2 a = unpack2(acc);
    a.x = fmaf(partial(p0, kFp8), __fmul_rn(sx, w0), a.x);
    a.y = fmaf(partial(p1, kFp8), __fmul_rn(sx, w1), a.y);
    acc = pack2(a.x, a.y);
  }
}

template <int kMode, bool kFp8, bool kPacked, bool kLR>
__global__ void __launch_bounds__(kThreads, 1)
    w4a4_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_ws, GemmEpilogue ep, int M, int N, int K,
                     uint32_t a_signed, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // row tiles vary fastest: the CTAs that run together share their weight tile (read from HBM about once)
  const int m_tile = blockIdx.x, n_tile = blockIdx.y;
  const int G = K / GROUP, KT = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
      mbar_init(&sm.ws_empty[s], 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 8);
    }
    mbar_init(&sm.mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensor_map(&map_a);
    prefetch_tensor_map(&map_b);
    prefetch_tensor_map(&map_ws);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp < 4) {
    setmaxnreg_dec<56>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&sm.empty[s], ph ^ 1, err, kErrWaitEmpty)) break;
        if (!mbar_wait(&sm.ws_empty[s], ph ^ 1, err, kErrWaitScale)) break;
        mbar_arrive_expect_tx(&sm.full[s], A_BYTES + B_BYTES + WS_BYTES);
        tma_load_2d(sm.a[s], &map_a, &sm.full[s], kt * BK, m_tile * BM);
        tma_load_2d(sm.b[s], &map_b, &sm.full[s], kt * BK, n_tile * BN);
        tma_load_2d(&sm.ws[s][0][0], &map_ws, &sm.full[s], n_tile * BN, kt * GPS);
        issued = kt + 1;
      }
      // Copies still in flight must land before the CTA exits; on the normal path they all have been consumed.
      for (int kt = (issued > STAGES ? issued - STAGES : 0); kt < issued; ++kt)
        mbar_wait(&sm.full[kt % STAGES], (kt / STAGES) & 1, err, kErrWaitFull);
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      // E4M3-coded operands: kind::f8f6f4 (e4m3 x e4m3 -> f32); int8 codes: kind::i8 (s8/u8 x s8 -> s32)
      const uint32_t idesc = kFp8 ? make_idesc(1, 0, 0, BM, BN) : make_idesc(2, a_signed, 1, BM, BN);
      bool ok = true;
      int g = 0;
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.full[s], ph, err, kErrWaitFull));
        if (!ok) break;
        tc_fence_after();
        for (int sub = 0; sub < GPS; ++sub, ++g) {
          const int b = g & 1;
          ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_empty[b], ((g >> 1) & 1) ^ 1, err, kErrWaitAccEmpty));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t a0 = smem_u32(sm.a[s]) + sub * GROUP;
            const uint32_t b0 = smem_u32(sm.b[s]) + sub * GROUP;
#pragma unroll
            for (int kk = 0; kk < GROUP / 32; ++kk)
              if constexpr (kFp8)
                mma_f8(tmem + b * BN, smem_desc_k128(a0 + kk * 32), smem_desc_k128(b0 + kk * 32), idesc, kk > 0);
              else
                mma_i8(tmem + b * BN, smem_desc_k128(a0 + kk * 32), smem_desc_k128(b0 + kk * 32), idesc, kk > 0);
            tc_commit(&sm.acc_full[b]);
          }
          __syncwarp();
        }
        if (ok) {
          if (elect_one()) tc_commit(&sm.empty[s]);
          __syncwarp();
        }
      }
      // All MMAs issued above have finished once this commit arrives (TMEM may be freed afterwards).
      if (elect_one()) tc_commit(&sm.mma_done);
      __syncwarp();
      mbar_wait(&sm.mma_done, 0, err, kErrWaitAccFull);
    }
  } else {
    setmaxnreg_inc<224>();
    // ---------------- promotion + epilogue ----------------
    const int q = warp & 3, h = (warp - 4) >> 2;
    const int row = q * 32 + lane;
    const int m = m_tile * BM + row;
    const bool row_ok = m < M;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + h * 128;
    uint64_t acc2[64];  // 128 fp32 accumulators as 64 column pairs
#pragma unroll
    for (int j = 0; j < 64; ++j) acc2[j] = 0ull;

    // sx[g, m], loaded kAhead groups ahead through a ring of registers: a group lasts well under the latency of
    // a load that misses L2, and the promotion of every element waits on it
    constexpr int kAhead = 4;
    float sxr[kAhead];
#pragma unroll
    for (int i = 0; i < kAhead; ++i) sxr[i] = row_ok && i < G ? __ldg(ep.ascale + static_cast<size_t>(i) * M + m) : 0.f;
    bool ok = true;
    for (int g = 0; g < G; ++g) {
      const int b = g & 1, kt = g / GPS, s = kt % STAGES, sub = g % GPS;
      const uint64_t sx2 = pack2(sxr[0], sxr[0]);
#pragma unroll
      for (int i = 0; i + 1 < kAhead; ++i) sxr[i] = sxr[i + 1];
      sxr[kAhead - 1] = row_ok && g + kAhead < G ? __ldg(ep.ascale + static_cast<size_t>(g + kAhead) * M + m) : 0.f;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_full[b], (g >> 1) & 1, err, kErrWaitAccFull));
      if (!ok) break;
      tc_fence_after();
      // the weight scales of this stage arrived with its tiles (full[s]); the MMA having run implies it, the
      // wait below makes the TMA's shared-memory writes visible to this thread
      if (sub == 0) {
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.full[s], (kt / STAGES) & 1, err, kErrWaitFull));
        if (!ok) break;
      }
      const uint32_t ws = smem_u32(&sm.ws[s][sub][h * 128]);
      const uint32_t t_buf = t_row + b * BN;
      // Drain the group's 128 columns in 4 chunks of 32, loading chunk c + 1 while chunk c is promoted.
      uint32_t ra[32], rb[32];
      tmem_ld32(t_buf, ra);
      tmem_ld_wait(ra);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t(&cur)[32] = (c & 1) ? rb : ra;
        uint32_t(&nxt)[32] = (c & 1) ? ra : rb;
        if (c < 3) tmem_ld32(t_buf + (c + 1) * 32, nxt);
        if (c == 3) {  // every column of this buffer is in registers: the MMA may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
        }
        if constexpr (kMode == kEpiDumpGroup) {
          if (g == ep.dump_group && row_ok) {
            int32_t* o = reinterpret_cast<int32_t*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n_tile * BN +
                         h * 128 + c * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = kFp8 ? __float2int_rn(__uint_as_float(cur[j])) : static_cast<int32_t>(cur[j]);
          }
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 w = lds128(ws + (c * 32 + j) * 4);
          promote2<kFp8, kPacked>(acc2[(c * 32 + j) / 2], cur[j], cur[j + 1], w.x, w.y, sx2);
          promote2<kFp8, kPacked>(acc2[(c * 32 + j) / 2 + 1], cur[j + 2], cur[j + 3], w.z, w.w, sx2);
        }
        if (c < 3) tmem_ld_wait(nxt);
      }
      if (sub == GPS - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.ws_empty[s]);
      }
    }
    float acc[128];
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float2 v = unpack2(acc2[j]);
      acc[2 * j] = v.x;
      acc[2 * j + 1] = v.y;
    }

    if (ok && row_ok) {
      const int n0 = n_tile * BN + h * 128;
      add_addend<128>(ep, m, n0, acc);
      if constexpr (kLR) add_lowrank<128>(ep, m, n0, acc);  // its own instantiations (registers)
      if constexpr (kMode == kEpiBf16) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
#pragma unroll
        for (int j = 0; j < 128; j += 8) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = acc[j + i] + (ep.bias ? __ldg(ep.bias + n0 + j + i) : 0.f);
          uint4 pk;
          __nv_bfloat162 t0 = __floats2bfloat162_rn(v[0], v[1]), t1 = __floats2bfloat162_rn(v[2], v[3]);
          __nv_bfloat162 t2 = __floats2bfloat162_rn(v[4], v[5]), t3 = __floats2bfloat162_rn(v[6], v[7]);
          pk.x = *reinterpret_cast<uint32_t*>(&t0);
          pk.y = *reinterpret_cast<uint32_t*>(&t1);
          pk.z = *reinterpret_cast<uint32_t*>(&t2);
          pk.w = *reinterpret_cast<uint32_t*>(&t3);
          *reinterpret_cast<uint4*>(out + j) = pk;
        }
      } else if constexpr (kMode == kEpiGeluU4) {
        // the fused MLP's hidden layer (reference quantization/w4a4.py:195-204, native/ops/w4a4_ops.cpp:44-63):
        // u = GELU(acc + bias) + shift (>= 0), divided by the next layer's smoothing, quantized unsigned per group
        // of 64 columns: scale = max(max u, 1e-8) / 15, code = round-half-even(u / scale) clamped to [0, 15]
        uint8_t* codes = reinterpret_cast<uint8_t*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
#pragma unroll
        for (int g2 = 0; g2 < 2; ++g2) {
          float u[64];
          float amax = 0.f;
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const int n = n0 + g2 * 64 + j;
            const float gv = gelu_tanh(acc[g2 * 64 + j] + (ep.bias ? __ldg(ep.bias + n) : 0.f));
            if (ep.gelu_out) ep.gelu_out[static_cast<size_t>(m) * ep.ld_gelu + n] = gv;
            float t = __fadd_rn(gv, ep.gelu_shift);
            if (ep.out_smooth) t = __fdiv_rn(t, __bfloat162float(ep.out_smooth[n]));
            u[j] = t;
            amax = fmaxf(amax, fabsf(t));
          }
          const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 15.f);
          const float rcp = __frcp_rn(scale);
#pragma unroll
          for (int j = 0; j < 64; j += 16) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint32_t word = 0;
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const int q = max(0, min(15, __float2int_rn(div_rn_by(u[j + e * 4 + b], scale, rcp))));
                word |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(static_cast<float>(q), __NV_SATFINITE, __NV_E4M3))
                        << (8 * b);
              }
              w[e] = word;
            }
            *reinterpret_cast<uint4*>(codes + g2 * 64 + j) = make_uint4(w[0], w[1], w[2], w[3]);
          }
          ep.out_scales[static_cast<size_t>((n0 + g2 * 64) / 64) * M + m] =
              ep.out_scale_dtype == 1 ? __half2float(__float2half_rn(scale)) : bf16_round(scale);
        }
      } else if constexpr (kMode == kEpiResidualF32) {
        // residual stream update in fp32: x_new = x + float(bf16(acc + bias)) * gate   (gate 1 when absent)
        float* out = reinterpret_cast<float*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
        // without a residual: the fp32 partial product acc (+ bias) of a row-parallel shard, unrounded
        const float* res = ep.residual ? ep.residual + static_cast<size_t>(m) * ep.ld_res + n0 : nullptr;
#pragma unroll
        for (int j = 0; j < 128; j += 4) {
          const float4 r = res ? *reinterpret_cast<const float4*>(res + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          float v[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p = acc[j + i] + (ep.bias ? __ldg(ep.bias + n0 + j + i) : 0.f);
            const float o = bf16_round(p);
            v[i] = !res ? p : ep.gate ? __fadd_rn(v[i], __fmul_rn(o, __ldg(ep.gate + n0 + j + i))) : __fadd_rn(v[i], o);
          }
          *reinterpret_cast<float4*>(out + j) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host side

static bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                        uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode_tiled(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int gemm_validate(const GemmArgs& a, const char** why) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) {
    *why = "M, N and K must be positive";
    return 1;
  }
  if (a.N % BN != 0) {
    *why = "N must be a multiple of 256";
    return 1;
  }
  if (a.K % BK != 0) {
    *why = "K must be a multiple of 128";
    return 1;
  }
  if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.b) | reinterpret_cast<uintptr_t>(a.wscale)) &
      15) {
    *why = "operand pointers must be 16-byte aligned";
    return 1;
  }
  return 0;
}

int gemm_launch(const GemmArgs& a, cudaStream_t stream, const char** why) {
  if (gemm_validate(a, why) != 0) return 1;
  CUtensorMap ma, mb, mw;
  if (!make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.a, a.K, a.M, a.lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.b, a.K, a.N, a.ldb, BK, BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.wscale, a.N, a.K / GROUP, static_cast<uint64_t>(a.N) * 4,
                   BN, GPS, CU_TENSOR_MAP_SWIZZLE_NONE)) {
    *why = "cuTensorMapEncodeTiled rejected an operand (alignment or stride)";
    return 2;
  }
  const dim3 grid((a.M + BM - 1) / BM, a.N / BN);
  cudaError_t e = cudaSuccess;
  auto launch = [&](auto kernel) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    if (e == cudaSuccess) kernel<<<grid, kThreads, kSmemBytes, stream>>>(ma, mb, mw, a.ep, a.M, a.N, a.K, a.a_signed, a.err);
  };
  const bool fp8 = a.code_format == kCodesE4M3;
  const bool packed = a.variant == 1;
  switch (a.ep.mode * 4 + (fp8 ? 2 : 0) + (packed ? 1 : 0)) {
#define WDL_GEMM_CASE(MODE, FP8, PACKED) \
  case MODE * 4 + (FP8 ? 2 : 0) + (PACKED ? 1 : 0):                                                         \
    a.ep.lr_act ? launch(w4a4_gemm_kernel<MODE, FP8, PACKED, true>) : launch(w4a4_gemm_kernel<MODE, FP8, PACKED, false>); \
    break;
    WDL_GEMM_CASE(kEpiBf16, false, false)
    WDL_GEMM_CASE(kEpiBf16, false, true)
    WDL_GEMM_CASE(kEpiBf16, true, false)
    WDL_GEMM_CASE(kEpiBf16, true, true)
    WDL_GEMM_CASE(kEpiResidualF32, false, false)
    WDL_GEMM_CASE(kEpiResidualF32, false, true)
    WDL_GEMM_CASE(kEpiResidualF32, true, false)
    WDL_GEMM_CASE(kEpiResidualF32, true, true)
    WDL_GEMM_CASE(kEpiDumpGroup, false, false)
    WDL_GEMM_CASE(kEpiDumpGroup, false, true)
    WDL_GEMM_CASE(kEpiDumpGroup, true, false)
    WDL_GEMM_CASE(kEpiDumpGroup, true, true)
    WDL_GEMM_CASE(kEpiGeluU4, true, false)
    WDL_GEMM_CASE(kEpiGeluU4, true, true)
#undef WDL_GEMM_CASE
    default: *why = "unknown epilogue mode"; return 1;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return 3;
  }
  return 0;
}

}  // namespace w4a4
}  // namespace wdl
