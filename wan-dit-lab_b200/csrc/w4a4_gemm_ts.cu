// W4A4 GEMM with the group-scale products on the tensor core (code format "E4M3, padded scales").
//
//   y[m, n] = sum_g  S_g[m, n] * P_g[m, n],    S_g[m, n] = sx[g, m] * sw[g, n],
//   P_g[m, n] = sum_{k in group g} xq[m, k] * wq[n, k]
//
// the arithmetic of SVDQuant's INT4 linear (Nunchaku's gemm_w4a4, called from the reference's
// native/ops/w4a4_ops.cpp:36): exact integer group partials, promoted by the product of the two group scales.
// Promoting on the CUDA cores costs a multiply (sx * sw) and a fused multiply-add per element and group: twice
// the tensor-core time of the group's MMA at the 8-bit rate, so that kernel (w4a4_gemm.cu) cannot pass half of
// the tensor peak. Here the tensor core also forms S_g: a rank-1 tf32 MMA (K = 8, the scales in column 0, zeros
// elsewhere) writes sx[g, m] * sw[g, n] into TMEM next to P_g. The product of a bf16 or f16 scale and a bf16
// or f16 scale has at most 22 significant bits, so it is exact in tf32 x tf32 -> f32, bit-identical to the
// CUDA-core multiply. The epilogue then does one FMA per element and group: acc = fma(P_g, S_g, acc), the same
// roundings in the same order as the CUDA-core promotion.
//
// Operands: codes are E4M3 bytes of the 4-bit integers (exact for [-8, 15]; kind::f8f6f4 leaves P_g as exact
// float32 integers). Scales are stored padded for the tensor core: [K / 64][rows][4] float32 holding
// (s, 0, 0, 0), so that the 128 rows of a tile, 2048 contiguous bytes, land by one bulk copy as the first K-half
// (4 tf32 columns) of a K-major no-swizzle operand; the second K-half is a block of zeros written once. (A
// tensor-map box of 128 rows x 16 bytes moves the same bytes row by row, and measured at less than half the
// GEMM's throughput.)
//
// Tile 128 x 128, two groups per pipeline stage, one CTA per SM, 12 warps:
//   warp 0      TMA producer: A, B code tiles (128-byte swizzle) and the four scale blocks of the stage
//   warp 1      TMEM owner and MMA issuer: per group 2 x K=32 f8f6f4 MMAs into P[g % 2], 1 tf32 MMA into S[g % 2]
//   warps 4-11  epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and columns 64 ((w - 4) / 4)
//               .. +63 of P and S, keeps 64 fp32 accumulators per thread
// TMEM: P[2] at columns 0 and 128, S[2] at 256 and 384 (all 512 columns).
#include "common.cuh"
#include "w4a4_gemm.h"

namespace wdl {
namespace w4a4 {
namespace ts {

constexpr int BM = 128, BN = 128, BK = 128, STAGES = 4, GROUP = 64;
constexpr int GPS = BK / GROUP;               // groups per stage
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
constexpr int SCALE_BLOCK = 4096;             // 128 rows x 8 tf32: data half (TMA) + zero half
constexpr int SCALE_DATA = 2048;              // 128 rows x 16 bytes
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) Smem {
  // the scale operand blocks come first: every descriptor built on them points inside this structure
  uint8_t sa[STAGES][GPS][SCALE_BLOCK];
  uint8_t sb[STAGES][GPS][SCALE_BLOCK];
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// Descriptor of a K-major operand in the no-swizzle canonical layout: 8-row core matrices of 16-byte rows,
// contiguous (128 bytes each); the next 8 rows 128 bytes further (stride byte offset), the next 16 bytes of K
// 2048 bytes further (leading byte offset: the zero half of the block).
__device__ __forceinline__ uint64_t smem_desc_scales(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(SCALE_DATA >> 4) << 16;  // leading byte offset: K direction
  d |= static_cast<uint64_t>(128u >> 4) << 32;        // stride byte offset: 8-row groups
  d |= static_cast<uint64_t>(1u) << 46;                // descriptor version for sm_100
  return d;                                            // layout type 0: no swizzle
}

// D[tmem] = A * B^T with tf32 operands and an f32 accumulator.
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// acc[j] = fma(P[j], S[j], acc[j]) for the 32 columns of one TMEM chunk.
__device__ __forceinline__ void promote32(float (&acc)[64], int base, const uint32_t (&p)[32], const uint32_t (&s)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[base + j] = fmaf(__uint_as_float(p[j]), __uint_as_float(s[j]), acc[base + j]);
}

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_ts_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const float* __restrict__ wscale, GemmEpilogue ep, int M, int N, int K, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // row tiles vary fastest: the CTAs that run together share their weight tile (read from HBM about once)
  const int m_tile = blockIdx.x, n_tile = blockIdx.y;
  const int G = K / GROUP, KT = K / BK;

  // zero halves of the scale blocks (never written again), made visible to the tensor core's proxy
  for (int i = threadIdx.x; i < STAGES * GPS * (SCALE_BLOCK - SCALE_DATA) / 16; i += kThreads) {
    const int blk = i / ((SCALE_BLOCK - SCALE_DATA) / 16), off = i % ((SCALE_BLOCK - SCALE_DATA) / 16);
    const int s = blk / GPS, sub = blk % GPS;
    *reinterpret_cast<uint4*>(&sm.sa[s][sub][SCALE_DATA + off * 16]) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(&sm.sb[s][sub][SCALE_DATA + off * 16]) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
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
      // activation scale rows of this tile: 128, or fewer in the last group of the last row tile (rows past
      // G * M do not exist; the rows of the next group that a partial tile reads feed only rows >= M)
      const int64_t a_rows_total = static_cast<int64_t>(G) * M;
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&sm.empty[s], ph ^ 1, err, kErrWaitEmpty)) break;
        uint32_t a_bytes[GPS];
        uint32_t tx = A_BYTES + B_BYTES + GPS * SCALE_DATA;
#pragma unroll
        for (int sub = 0; sub < GPS; ++sub) {
          const int64_t row0 = static_cast<int64_t>(kt * GPS + sub) * M + m_tile * BM;
          const int64_t rows = a_rows_total - row0 < BM ? a_rows_total - row0 : BM;
          a_bytes[sub] = static_cast<uint32_t>(rows) * 16u;
          tx += a_bytes[sub];
        }
        mbar_arrive_expect_tx(&sm.full[s], tx);
        tma_load_2d(sm.a[s], &map_a, &sm.full[s], kt * BK, m_tile * BM);
        tma_load_2d(sm.b[s], &map_b, &sm.full[s], kt * BK, n_tile * BN);
#pragma unroll
        for (int sub = 0; sub < GPS; ++sub) {
          const int g = kt * GPS + sub;
          bulk_load(sm.sa[s][sub], ep.ascale + (static_cast<int64_t>(g) * M + m_tile * BM) * 4, a_bytes[sub],
                    &sm.full[s]);
          bulk_load(sm.sb[s][sub], wscale + (static_cast<int64_t>(g) * N + n_tile * BN) * 4, SCALE_DATA,
                    &sm.full[s]);
        }
        issued = kt + 1;
      }
      for (int kt = (issued > STAGES ? issued - STAGES : 0); kt < issued; ++kt)
        mbar_wait(&sm.full[kt % STAGES], (kt / STAGES) & 1, err, kErrWaitFull);
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc_p = make_idesc(1, 0, 0, BM, BN);  // e4m3 x e4m3 -> f32
      const uint32_t idesc_s = make_idesc(1, 2, 2, BM, BN);  // tf32 x tf32 -> f32
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
            mma_f8(tmem + b * BN, smem_desc_k128(a0), smem_desc_k128(b0), idesc_p, 0u);
            mma_f8(tmem + b * BN, smem_desc_k128(a0 + 32), smem_desc_k128(b0 + 32), idesc_p, 1u);
            mma_tf32(tmem + 2 * BN + b * BN, smem_desc_scales(smem_u32(sm.sa[s][sub])),
                     smem_desc_scales(smem_u32(sm.sb[s][sub])), idesc_s);
            tc_commit(&sm.acc_full[b]);
          }
          __syncwarp();
        }
        if (ok) {
          if (elect_one()) tc_commit(&sm.empty[s]);
          __syncwarp();
        }
      }
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
    const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + h * 64;
    float acc[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;

    bool ok = true;
    for (int g = 0; g < G; ++g) {
      const int b = g & 1;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_full[b], (g >> 1) & 1, err, kErrWaitAccFull));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tp = t_row + b * BN, ts = t_row + 2 * BN + b * BN;
      // all four loads in flight at once, one wait, then the buffer pair goes back to the MMA issuer before any
      // arithmetic: the release comes one TMEM round trip after the commit
      uint32_t p0[32], s0[32], p1[32], s1[32];
      tmem_ld32(tp, p0);
      tmem_ld32(ts, s0);
      tmem_ld32(tp + 32, p1);
      tmem_ld32(ts + 32, s1);
      tmem_ld_wait(p0);
      tmem_ld_wait(s0);
      tmem_ld_wait(p1);
      tmem_ld_wait(s1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
      if constexpr (kMode == kEpiDumpGroup) {
        if (g == ep.dump_group && row_ok) {
          int32_t* o = reinterpret_cast<int32_t*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n_tile * BN + h * 64;
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float2int_rn(__uint_as_float(p0[j]));
#pragma unroll
          for (int j = 0; j < 32; ++j) o[32 + j] = __float2int_rn(__uint_as_float(p1[j]));
        }
      }
      promote32(acc, 0, p0, s0);
      promote32(acc, 32, p1, s1);
    }

    if (ok && row_ok) {
      const int n0 = n_tile * BN + h * 64;
      add_addend<64>(ep, m, n0, acc);
      if constexpr (kMode == kEpiBf16) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
#pragma unroll
        for (int j = 0; j < 64; j += 8) {
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
        // u = GELU(acc + bias) + shift, divided by the next layer's smoothing, quantized unsigned per group of
        // 64 columns (this thread's 64 columns are one group): scale = max(max u, 1e-8) / 15, code =
        // round-half-even(u / scale) clamped to [0, 15], stored as E4M3 bytes; the scale in the padded layout.
        uint8_t* codes = reinterpret_cast<uint8_t*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const int n = n0 + j;
          const float gv = gelu_tanh(acc[j] + (ep.bias ? __ldg(ep.bias + n) : 0.f));
          if (ep.gelu_out) ep.gelu_out[static_cast<size_t>(m) * ep.ld_gelu + n] = gv;
          float t = __fadd_rn(gv, ep.gelu_shift);
          if (ep.out_smooth) t = __fdiv_rn(t, __bfloat162float(ep.out_smooth[n]));
          acc[j] = t;
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
            for (int i = 0; i < 4; ++i) {
              const int c = max(0, min(15, __float2int_rn(div_rn_by(acc[j + e * 4 + i], scale, rcp))));
              word |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(static_cast<float>(c), __NV_SATFINITE, __NV_E4M3))
                      << (8 * i);
            }
            w[e] = word;
          }
          *reinterpret_cast<uint4*>(codes + j) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        const float stored = ep.out_scale_dtype == 1 ? __half2float(__float2half_rn(scale)) : bf16_round(scale);
        *reinterpret_cast<float4*>(ep.out_scales + (static_cast<size_t>(n0 / 64) * M + m) * 4) =
            make_float4(stored, 0.f, 0.f, 0.f);
      } else if constexpr (kMode == kEpiResidualF32) {
        float* out = reinterpret_cast<float*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
        // without a residual: the fp32 partial product acc (+ bias) of a row-parallel shard, unrounded
        const float* res = ep.residual ? ep.residual + static_cast<size_t>(m) * ep.ld_res + n0 : nullptr;
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
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

}  // namespace ts

int gemm_ts_validate(const GemmArgs& a, const char** why) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) {
    *why = "M, N and K must be positive";
    return 1;
  }
  if (a.N % ts::BN != 0) {
    *why = "N must be a multiple of 128";
    return 1;
  }
  if (a.K % ts::BK != 0) {
    *why = "K must be a multiple of 128";
    return 1;
  }
  if (static_cast<int64_t>(a.K / ts::GROUP) * (a.M > a.N ? a.M : a.N) > (int64_t{1} << 31) - 1) {
    *why = "K / 64 * max(M, N) must fit in 31 bits";
    return 1;
  }
  if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.b) | reinterpret_cast<uintptr_t>(a.wscale) |
       reinterpret_cast<uintptr_t>(a.ep.ascale)) & 15) {
    *why = "operand and scale pointers must be 16-byte aligned";
    return 1;
  }
  if (a.ep.mode == kEpiGeluU4 && (reinterpret_cast<uintptr_t>(a.ep.out_scales) & 15)) {
    *why = "out_scales must be 16-byte aligned";
    return 1;
  }
  return 0;
}

int gemm_ts_launch(const GemmArgs& a, cudaStream_t stream, const char** why) {
  if (gemm_ts_validate(a, why) != 0) return 1;
  CUtensorMap ma, mb;
  if (!ts::make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.a, a.K, a.M, a.lda, ts::BK, ts::BM,
                       CU_TENSOR_MAP_SWIZZLE_128B) ||
      !ts::make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.b, a.K, a.N, a.ldb, ts::BK, ts::BN,
                       CU_TENSOR_MAP_SWIZZLE_128B)) {
    *why = "cuTensorMapEncodeTiled rejected an operand (alignment or stride)";
    return 2;
  }
  const dim3 grid((a.M + ts::BM - 1) / ts::BM, a.N / ts::BN);
  cudaError_t e = cudaSuccess;
  auto launch = [&](auto kernel) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ts::kSmemBytes));
    if (e == cudaSuccess)
      kernel<<<grid, ts::kThreads, ts::kSmemBytes, stream>>>(ma, mb, a.wscale, a.ep, a.M, a.N, a.K, a.err);
  };
  switch (a.ep.mode) {
    case kEpiBf16: launch(ts::gemm_ts_kernel<kEpiBf16>); break;
    case kEpiResidualF32: launch(ts::gemm_ts_kernel<kEpiResidualF32>); break;
    case kEpiDumpGroup: launch(ts::gemm_ts_kernel<kEpiDumpGroup>); break;
    case kEpiGeluU4: launch(ts::gemm_ts_kernel<kEpiGeluU4>); break;
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
