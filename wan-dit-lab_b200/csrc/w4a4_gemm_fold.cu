// W4A4 GEMM with the weight group scales folded into 16-bit weights (code format "f16 fold").
//
//   y[m, n] = sum_g  sx[g, m] * (sw[g, n] * P_g[m, n]),   P_g[m, n] = sum_{k in group g} xq[m, k] * wq[n, k]
//
// SVDQuant's INT4 linear (Nunchaku's gemm_w4a4, called from the reference's native/ops/w4a4_ops.cpp:36). The
// promotion of the INT4 kernels multiplies each exact group partial by sx * sw: two float32 operations per
// accumulator element and group on the CUDA cores, twice the tensor-core time of the group. Here the weight
// scale travels with the weight instead. With bf16 weight scales (the repo's packing, w4a4.py:177) every
// product wq * sw has at most 3 + 8 = 11 significant bits, so it is an exact float16 number once the layer is
// shifted by one power of two 2^-F into float16's normal range (wdl_w4a4_fold_weight checks every element and
// reports any that is not exact). The activation codes are exact float16 integers. A kind::f16 tcgen05.mma of
// codes x folded weights then accumulates, for each group, sw[g, n] * 2^-F * P_g[m, n]: every partial sum is an
// integer (|P| <= 4096, 13 bits) times sw (8 bits), 21 significant bits, exact in float32 in any order. The
// epilogue adds it with ONE fused multiply-add by the per-row scalar sx[g, m] * 2^F:
//   acc = fma(sw 2^-F P, sx 2^F, acc) = round(acc + sx sw P),
// the same rounding of the same exact product as the CUDA-core promotion fma(P, sx * sw, acc) (sx * sw is exact
// too), so results equal the E4M3 / int8 kernels' bit for bit. The price is the 16-bit tensor rate (half the
// 8-bit rate) and 2-byte operands; the CUDA cores, which bound the other kernels, do half the work and no
// shared-memory scale loads.
//
// Tile 128 x 256, one group (64 k = 128 bytes of a row) per pipeline stage, 4 stages, one CTA per SM, 12 warps:
//   warp 0      TMA producer: A, B tiles (128-byte swizzle)
//   warp 1      TMEM owner and MMA issuer: 4 x K=16 kind::f16 MMAs per group into TMEM buffer (group % 2)
//   warps 4-11  promotion + epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and columns
//               128 ((w - 4) / 4) .. +127, keeps 128 fp32 accumulators per thread
// TMEM: 2 buffers x 256 columns = all 512.
//
// gemm_pre_kernel (further down) takes the prescaled activations of kCodesF16Pre instead, whose products carry
// both scales: it accumulates all of K per tile and runs persistently (one CTA per SM, two TMEM accumulators),
// finishing each tile behind the next tile's main loop. Both kernels share the tile epilogue (finish_tile).
#include "common.cuh"
#include "w4a4_gemm.h"

namespace wdl {
namespace w4a4 {
namespace fold {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) Smem {
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

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// The end of a tile for one epilogue thread: row m_tile * BM + 32 q + lane of the 128 columns n_tile * BN + 128 h
// .. + 127 in acc (the finished fp32 products): the low-rank branch (an addend or its up-projection), then the
// mode's epilogue. tw: this warp's
// 32 x 33 floats of shared-memory scratch (residual mode).
template <int kMode, bool kLR>
__device__ __forceinline__ void finish_tile(float (&acc)[128], const GemmEpilogue& ep, float* tw, int M, int N,
                                            int m_tile, int n_tile, int q, int h, int lane, bool ok) {
  const int row = q * 32 + lane;
  const int m = m_tile * BM + row;
  const bool row_ok = m < M;
  // N % 128 == 0: the last column tile may hold only its first half (the TMA zero-fills the missing weight rows)
  const bool col_ok = n_tile * BN + h * 128 < N;
  if (ok && row_ok && col_ok) {
    add_addend<128>(ep, m, n_tile * BN + h * 128, acc);
    if constexpr (kLR) add_lowrank<128>(ep, m, n_tile * BN + h * 128, acc);  // its own instantiations (registers)
  }

  if constexpr (kMode == kEpiResidualF32) {
    // Residual update through a per-warp 32 x 32 transpose in shared memory (the pipeline buffers, idle once every
    // MMA has completed): lane l then owns column l of a 32-column block and the warp reads and writes whole rows
    // (128 contiguous bytes) instead of 32 rows at once, all 32 rows' loads in flight together; bias and gate are
    // loaded once per column. Same arithmetic per element as a thread-per-row update.
    const int m0 = m_tile * BM + q * 32;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
#pragma unroll
      for (int j = 0; j < 32; ++j) tw[lane * 33 + j] = acc[blk * 32 + j];
      __syncwarp();
      const int n = n_tile * BN + h * 128 + blk * 32 + lane;
      const float bn = ep.bias && col_ok ? __ldg(ep.bias + n) : 0.f;
      if (ok && col_ok && !ep.residual) {
        // a partial product in fp32 (a shard's share of a row-parallel layer, summed across shards before the
        // bias, rounding and residual update): out = acc (+ bias), no rounding
        float* out = reinterpret_cast<float*>(ep.out) + n;
#pragma unroll
        for (int r = 0; r < 32; ++r)
          if (m0 + r < M) out[static_cast<size_t>(m0 + r) * ep.ld_out] = tw[r * 33 + lane] + bn;
      } else if (ok && col_ok) {
        {
          // residual stream update in fp32: x_new = x + float(bf16(acc + bias)) * gate   (gate 1 when absent)
          const float gn = ep.gate ? __ldg(ep.gate + n) : 0.f;
          float* out = reinterpret_cast<float*>(ep.out) + n;
          const float* res = ep.residual + n;
          float x[32];  // all 32 rows' residuals in flight at once: unconditional loads (rows past M read the last
                        // row, their values unused), so that nothing holds one load back behind another
#pragma unroll
          for (int r = 0; r < 32; ++r) x[r] = res[static_cast<size_t>(min(m0 + r, M - 1)) * ep.ld_res];
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const float o = bf16_round(tw[r * 33 + lane] + bn);
            if (m0 + r < M)
              out[static_cast<size_t>(m0 + r) * ep.ld_out] = ep.gate ? __fadd_rn(x[r], __fmul_rn(o, gn)) : __fadd_rn(x[r], o);
          }
        }
      }
      __syncwarp();
    }
  }
  if (ok && row_ok && col_ok) {
    const int n0 = n_tile * BN + h * 128;
    if constexpr (kMode == kEpiBf16 || kMode == kEpiGeluU4) {
      // acc + bias before the mode's own work, the bias (16-byte aligned, checked by the callers) 16 bytes a load
      // (a scalar load per element inside the GELU loop made that epilogue 10 % slower). Without a bias acc + 0,
      // as the same sum with a zero bias (a -0 becomes +0).
      if (ep.bias) {
#pragma unroll
        for (int j = 0; j < 128; j += 4) {
          float4 b;  // loaded where used (hoisted, all 32 loads would be held in registers at once)
          asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(b.x), "=f"(b.y), "=f"(b.z), "=f"(b.w)
                       : "l"(ep.bias + n0 + j));
          acc[j] += b.x, acc[j + 1] += b.y, acc[j + 2] += b.z, acc[j + 3] += b.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 128; ++j) acc[j] += 0.f;
      }
    }
    if constexpr (kMode == kEpiBf16) {
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
#pragma unroll
      for (int j = 0; j < 128; j += 8) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = acc[j + i];
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
      // u = GELU(acc + bias) + shift, divided by the next layer's smoothing, quantized unsigned per group of 64
      // columns: scale = max(max u, 1e-8) / 15, code = round-half-even(u / scale) clamped to [0, 15], stored as
      // the next layer's float16 operand (exact integers) with the scale [N / 64, M] rounded to its dtype.
      uint16_t* codes = reinterpret_cast<uint16_t*>(ep.out) + static_cast<size_t>(m) * ep.ld_out + n0;
#pragma unroll
      for (int g2 = 0; g2 < 2; ++g2) {
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const int n = n0 + g2 * 64 + j;
          const float gv = gelu_tanh(acc[g2 * 64 + j]);
          if (ep.gelu_out) ep.gelu_out[static_cast<size_t>(m) * ep.ld_gelu + n] = gv;
          float t = __fadd_rn(gv, ep.gelu_shift);
          if (ep.out_smooth) t = __fdiv_rn(t, __bfloat162float(ep.out_smooth[n]));
          acc[g2 * 64 + j] = t;
          amax = fmaxf(amax, fabsf(t));
        }
        const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 15.f);
        const float rcp = __frcp_rn(scale);
#pragma unroll
        for (int j = 0; j < 64; j += 8) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // clamp to [0, 15], then round half to even by adding and subtracting 1.5 2^23 (exact below 2^22):
            // the codes of rint-then-clamp, without a conversion instruction; two per float16 pack
            float r2[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const float d = fminf(fmaxf(div_rn_by(acc[g2 * 64 + j + 2 * e + t], scale, rcp), 0.f), 15.f);
              r2[t] = __fsub_rn(__fadd_rn(d, 12582912.f), 12582912.f);
            }
            const __half2 hp = __floats2half2_rn(r2[0], r2[1]);
            w[e] = *reinterpret_cast<const uint32_t*>(&hp);
          }
          *reinterpret_cast<uint4*>(codes + g2 * 64 + j) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        ep.out_scales[static_cast<size_t>((n0 + g2 * 64) / 64) * M + m] =
            ep.out_scale_dtype == 1 ? __half2float(__float2half_rn(scale)) : bf16_round(scale);
      }
    }
  }
}

template <int kMode, bool kLR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_fold_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const float* __restrict__ fold_scale, GemmEpilogue ep, int M, int N, int K, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // row tiles vary fastest: the CTAs that run together share their weight tile (read from HBM about once)
  const int m_tile = blockIdx.x, n_tile = blockIdx.y;
  const int G = K / BK;

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
      int issued = 0;
      for (int g = 0; g < G; ++g) {
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1;
        if (!mbar_wait(&sm.empty[s], ph ^ 1, err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&sm.full[s], A_BYTES + B_BYTES);
        tma_load_2d(sm.a[s], &map_a, &sm.full[s], g * BK, m_tile * BM);
        tma_load_2d(sm.b[s], &map_b, &sm.full[s], g * BK, n_tile * BN);
        issued = g + 1;
      }
      for (int g = (issued > STAGES ? issued - STAGES : 0); g < issued; ++g)
        mbar_wait(&sm.full[g % STAGES], (g / STAGES) & 1, err, kErrWaitFull);
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = make_idesc(1, 0, 0, BM, BN);  // f16 x f16 -> f32
      bool ok = true;
      for (int g = 0; g < G && ok; ++g) {
        const int s = g % STAGES, b = g & 1;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.full[s], (g / STAGES) & 1, err, kErrWaitFull)) &&
             __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_empty[b], ((g >> 1) & 1) ^ 1, err, kErrWaitAccEmpty));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t a0 = smem_u32(sm.a[s]), b0 = smem_u32(sm.b[s]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16(tmem + b * BN, smem_desc_k128(a0 + kk * 32), smem_desc_k128(b0 + kk * 32), idesc, kk > 0);
          tc_commit(&sm.acc_full[b]);
          tc_commit(&sm.empty[s]);
        }
        __syncwarp();
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
    const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) + h * 128;
    const float unfold = __ldg(fold_scale);  // 2^F
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.f;

    bool ok = true;
    // sx[g, m], loaded kAhead groups ahead through a ring of registers: a group lasts well under the latency of
    // a load that misses L2, and the promotion of every element waits on it
    constexpr int kAhead = 4;
    float sxr[kAhead];
#pragma unroll
    for (int i = 0; i < kAhead; ++i)
      sxr[i] = row_ok && i < G ? __ldg(ep.ascale + static_cast<size_t>(i) * M + m) : 0.f;
    for (int g = 0; g < G; ++g) {
      const int b = g & 1;
      const float mul = __fmul_rn(sxr[0], unfold);  // sx * 2^F, exact: a power of two
#pragma unroll
      for (int i = 0; i + 1 < kAhead; ++i) sxr[i] = sxr[i + 1];
      sxr[kAhead - 1] = row_ok && g + kAhead < G ? __ldg(ep.ascale + static_cast<size_t>(g + kAhead) * M + m) : 0.f;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_full[b], (g >> 1) & 1, err, kErrWaitAccFull));
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_buf = t_row + b * BN;
      // Drain the group's 128 columns in two rounds of 64 (two 32-column loads in flight, one wait each round):
      // tcgen05.wait::ld waits for every load of the thread, so fewer, larger rounds expose its latency less.
      uint32_t ra[32], rb[32];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        tmem_ld32(t_buf + r * 64, ra);
        tmem_ld32(t_buf + r * 64 + 32, rb);
        tmem_ld_wait(ra);
        tmem_ld_wait(rb);
        if (r == 1) {  // every column of this buffer is in registers: the MMA may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[r * 64 + j] = fmaf(__uint_as_float(ra[j]), mul, acc[r * 64 + j]);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[r * 64 + 32 + j] = fmaf(__uint_as_float(rb[j]), mul, acc[r * 64 + 32 + j]);
      }
    }

    if constexpr (kMode == kEpiResidualF32) fence_proxy_async_smem();  // the scratch is a pipeline buffer
    finish_tile<kMode, kLR>(acc, ep, reinterpret_cast<float*>(sm.a[0]) + (warp - 4) * 32 * 33, M, N, m_tile, n_tile, q,
                       h, lane, ok);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- the prescaled format (kCodesF16Pre), persistent ------------------------------------------------------------
// With both scales folded into the operands, a tile is one plain accumulation over all of K: its accumulator
// (256 TMEM columns) is drained once, at the end. One CTA per SM loops over the tiles (tile t: m tile t % m_tiles,
// n tile t / m_tiles, so that the CTAs running together share weight tiles) with two accumulators: the MMA
// accumulates tile i + 1 into one while the epilogue warps drain tile i from the other and finish it (scale by
// 2^E_m 2^F, addend, bias, mode), so the epilogue is hidden behind the next tile's main loop. The TMA producer and
// the pipeline stages run on across tile boundaries. Same warp roles as gemm_fold_kernel; the residual mode's
// transposes use scratch of their own (the stages stay busy).
struct __align__(1024) SmemP {
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  float scratch[8][32 * 33];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
};

constexpr size_t kSmemPBytes = sizeof(SmemP) + 1024;

template <int kMode, bool kLR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pre_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const float* __restrict__ fold_scale, GemmEpilogue ep, int M, int N, int K, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  SmemP& sm = *reinterpret_cast<SmemP*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = K / BK;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;

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
      // ---------------- TMA producer: every k block of every tile of this CTA, through the ring of stages
      int kb = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m_tile = t % m_tiles, n_tile = t / m_tiles;
        for (int g = 0; g < G; ++g, ++kb) {
          const int s = kb % STAGES;
          if (!mbar_wait(&sm.empty[s], ((kb / STAGES) & 1) ^ 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[s], A_BYTES + B_BYTES);
          tma_load_2d(sm.a[s], &map_a, &sm.full[s], g * BK, m_tile * BM);
          tma_load_2d(sm.b[s], &map_b, &sm.full[s], g * BK, n_tile * BN);
        }
      }
      for (int j = (kb > STAGES ? kb - STAGES : 0); j < kb; ++j)  // no copy in flight at exit
        mbar_wait(&sm.full[j % STAGES], (j / STAGES) & 1, err, kErrWaitFull);
    } else if (warp == 1) {
      // ---------------- MMA issuer: tile i into accumulator i % 2, all of K
      const uint32_t idesc = make_idesc(1, 0, 0, BM, BN);  // f16 x f16 -> f32
      bool ok = true;
      int kb = 0, i = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int b = i & 1;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_empty[b], ((i >> 1) & 1) ^ 1, err, kErrWaitAccEmpty));
        if (!ok) break;
        tc_fence_after();
        for (int g = 0; g < G; ++g, ++kb) {
          const int s = kb % STAGES;
          ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.full[s], (kb / STAGES) & 1, err, kErrWaitFull));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t a0 = smem_u32(sm.a[s]), b0 = smem_u32(sm.b[s]);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_f16(tmem + b * BN, smem_desc_k128(a0 + kk * 32), smem_desc_k128(b0 + kk * 32), idesc,
                      g > 0 || kk > 0);
            tc_commit(&sm.empty[s]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) tc_commit(&sm.acc_full[b]);
        __syncwarp();
      }
      if (elect_one()) tc_commit(&sm.mma_done);
      __syncwarp();
      mbar_wait(&sm.mma_done, 0, err, kErrWaitAccFull);
    }
  } else {
    setmaxnreg_inc<224>();
    // ---------------- epilogue: drain tile i's accumulator, hand it back, finish the tile
    const int q = warp & 3, h = (warp - 4) >> 2;
    const float unfold = __ldg(fold_scale);  // 2^F
    float* tw = sm.scratch[warp - 4];
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int m_tile = t % m_tiles, n_tile = t / m_tiles;
      const int b = i & 1;
      const int m = m_tile * BM + q * 32 + lane;
      const float mul = __fmul_rn(m < M ? __ldg(ep.ascale + m) : 0.f, unfold);  // 2^E_m 2^F: exact
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_full[b], (i >> 1) & 1, err, kErrWaitAccFull))) break;
      tc_fence_after();
      const uint32_t t_buf = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN + h * 128;
      float acc[128];
      uint32_t ra[32], rb[32];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        tmem_ld32(t_buf + r * 64, ra);
        tmem_ld32(t_buf + r * 64 + 32, rb);
        tmem_ld_wait(ra);
        tmem_ld_wait(rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[r * 64 + j] = __fmul_rn(__uint_as_float(ra[j]), mul);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[r * 64 + 32 + j] = __fmul_rn(__uint_as_float(rb[j]), mul);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);  // every column in registers: the MMA may reuse the buffer
      finish_tile<kMode, kLR>(acc, ep, tw, M, N, m_tile, n_tile, q, h, lane, true);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- the prescaled format on CTA pairs (2-SM MMAs) ---------------------------------------------------------------
// gemm_pre_kernel is bound by how fast the TMA fills each SM's shared memory: a 128 x 256 x 64 step brings 48 KB
// (16 KB of activations, 32 KB of weights), about 650 SM cycles at the 71-81 B per cycle measured, against 512
// cycles of f16 MMA. Here a cluster of two CTAs (the two SMs of a TPC) computes 256 x 256 tiles with 2-SM MMAs
// (M = 256): each CTA holds its own 128 activation rows and one half (128 rows) of the weight tile, 32 KB a step,
// and the tensor cores of both SMs read both weight halves. Six stages of 32 KB per SM are in flight. Each CTA's
// TMEM holds its 128 rows of the accumulator, which its epilogue warps drain and finish as in gemm_pre_kernel
// (the same finish_tile). Roles:
//   both CTAs, warp 0      TMA producer of its own halves; every completion counts on the first CTA's full[s]
//   first CTA, warp 1      MMA issuer (one thread): 2-SM tcgen05.mma into accumulator (tile % 2), commits to its
//                          empty[s] / acc_full[b]; its producer relays empty[s] to the second CTA (remote arrive)
//   first CTA, warp 2      relays acc_full[b] to the second CTA
//   both CTAs, warps 4-11  epilogue; every warp of both CTAs arrives on the first CTA's acc_empty[b] (16 arrivals)
// Tiles: 256 rows x 256 columns, pair p takes tiles p, p + pairs, ... (row pairs fastest). No multicast is used.
constexpr int PSTAGES = 6;
constexpr int PA_BYTES = BM * BK * 2, PB_BYTES = (BN / 2) * BK * 2;  // per CTA and step: 16 KB + 16 KB

struct __align__(1024) SmemPair {
  uint8_t a[PSTAGES][PA_BYTES];
  uint8_t b[PSTAGES][PB_BYTES];
  float scratch[8][32 * 33];
  uint64_t full[PSTAGES];   // first CTA: both CTAs' halves of the step in stage s have landed
  uint64_t empty[PSTAGES];  // each CTA: its stage s may be refilled
  uint64_t acc_full[2];     // each CTA: accumulator b holds a finished tile
  uint64_t acc_empty[2];    // first CTA: accumulator b drained by the epilogues of both CTAs
  uint64_t mma_done;
  uint32_t tmem_base;
};

constexpr size_t kSmemPairBytes = sizeof(SmemPair) + 1024;
static_assert(kSmemPairBytes <= 232448, "shared memory of a CTA pair's stage ring");

template <int kMode, bool kLR>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pre_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const float* __restrict__ fold_scale, GemmEpilogue ep, int M, int N, int K, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  SmemPair& sm = *reinterpret_cast<SmemPair*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int G = K / BK;
  const int m_pairs = (M + 2 * BM - 1) / (2 * BM), n_tiles = (N + BN - 1) / BN;
  const int tiles = m_pairs * n_tiles;
  const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 16);
    }
    mbar_init(&sm.mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensor_map(&map_a);
    prefetch_tensor_map(&map_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(&sm.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialized before any remote arrive or copy completion reaches them
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp < 4) {
    setmaxnreg_dec<56>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer (both CTAs): this CTA's halves of every step, counted on the first CTA's full[s]
      const uint32_t full0 = peer_smem(smem_u32(&sm.full[0]), 0);
      const uint32_t peer_empty0 = peer_smem(smem_u32(&sm.empty[0]), 1);
      int kb = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        const int m_pair = t % m_pairs, n_tile = t / m_pairs;
        const int row0 = (m_pair * 2 + static_cast<int>(rank)) * BM;
        const int col0 = n_tile * BN + static_cast<int>(rank) * (BN / 2);
        for (int g = 0; g < G; ++g, ++kb) {
          const int s = kb % PSTAGES;
          if (!mbar_wait(&sm.empty[s], ((kb / PSTAGES) & 1) ^ 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 2 * (PA_BYTES + PB_BYTES));
          tma_load_2d_pair(sm.a[s], &map_a, full0 + 8 * s, g * BK, row0);
          tma_load_2d_pair(sm.b[s], &map_b, full0 + 8 * s, g * BK, col0);
          // the MMAs that read stage s (both CTAs' halves) have completed (their commit is what empty[s] waited
          // for): the second CTA may refill its half too. A relaxed arrive: nothing this thread wrote is handed over.
          if (rank == 0 && kb >= PSTAGES) mbar_arrive_cluster_relaxed(peer_empty0 + 8 * s);
        }
      }
      if (rank == 0)  // no copy of either CTA in flight at exit: both count on these barriers
        for (int j = (kb > PSTAGES ? kb - PSTAGES : 0); j < kb; ++j)
          mbar_wait(&sm.full[j % PSTAGES], (j / PSTAGES) & 1, err, kErrWaitFull);
    } else if (warp == 1 && rank == 0) {
      // ---------------- MMA issuer (first CTA): tile i into accumulator i % 2, all of K, 2-SM MMAs M = N = 256
      const uint32_t idesc = make_idesc(1, 0, 0, 2 * BM, BN);  // f16 x f16 -> f32
      bool ok = true;
      int kb = 0, i = 0;
      for (int t = pair; t < tiles && ok; t += pairs, ++i) {
        const int b = i & 1;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_empty[b], ((i >> 1) & 1) ^ 1, err, kErrWaitAccEmpty));
        if (!ok) break;
        tc_fence_after();
        for (int g = 0; g < G; ++g, ++kb) {
          const int s = kb % PSTAGES;
          ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.full[s], (kb / PSTAGES) & 1, err, kErrWaitFull));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t a0 = smem_u32(sm.a[s]), b0 = smem_u32(sm.b[s]);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_f16_pair(tmem + b * BN, smem_desc_k128(a0 + kk * 32), smem_desc_k128(b0 + kk * 32), idesc,
                           g > 0 || kk > 0);
            tc_commit_pair(&sm.empty[s]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) tc_commit_pair(&sm.acc_full[b]);
        __syncwarp();
      }
      if (elect_one()) tc_commit_pair(&sm.mma_done);
      __syncwarp();
      mbar_wait(&sm.mma_done, 0, err, kErrWaitAccFull);
    } else if (warp == 2 && rank == 0 && lane == 0) {
      // ---------------- relay (first CTA): accumulator b of tile i is complete in the second CTA's TMEM as well
      const uint32_t peer_acc_full0 = peer_smem(smem_u32(&sm.acc_full[0]), 1);
      int i = 0;
      for (int t = pair; t < tiles; t += pairs, ++i) {
        const int b = i & 1;
        if (!mbar_wait(&sm.acc_full[b], (i >> 1) & 1, err, kErrWaitAccFull)) break;
        mbar_arrive_cluster(peer_acc_full0 + 8 * b);
      }
    }
  } else {
    setmaxnreg_inc<224>();
    // ---------------- epilogue (both CTAs): drain this CTA's 128 rows of tile i, hand the buffer back, finish
    const int q = warp & 3, h = (warp - 4) >> 2;
    const float unfold = __ldg(fold_scale);  // 2^F
    float* tw = sm.scratch[warp - 4];
    const uint32_t acc_empty0 = peer_smem(smem_u32(&sm.acc_empty[0]), 0);
    int i = 0;
    for (int t = pair; t < tiles; t += pairs, ++i) {
      const int m_pair = t % m_pairs, n_tile = t / m_pairs;
      const int m_tile = m_pair * 2 + static_cast<int>(rank);  // this CTA's 128-row tile
      const int b = i & 1;
      const int m = m_tile * BM + q * 32 + lane;
      const float mul = __fmul_rn(m < M ? __ldg(ep.ascale + m) : 0.f, unfold);  // 2^E_m 2^F: exact
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sm.acc_full[b], (i >> 1) & 1, err, kErrWaitAccFull))) break;
      tc_fence_after();
      const uint32_t t_buf = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN + h * 128;
      float acc[128];
      uint32_t ra[32], rb[32];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        tmem_ld32(t_buf + r * 64, ra);
        tmem_ld32(t_buf + r * 64 + 32, rb);
        tmem_ld_wait(ra);
        tmem_ld_wait(rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[r * 64 + j] = __fmul_rn(__uint_as_float(ra[j]), mul);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[r * 64 + 32 + j] = __fmul_rn(__uint_as_float(rb[j]), mul);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * b);  // every column in registers: the MMA may reuse it
      finish_tile<kMode, kLR>(acc, ep, tw, M, N, m_tile, n_tile, q, h, lane, true);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other's MMAs, copies or remote arrives may still reach it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// Folded weights: w16[n, k] = float16(wq[n, k] * sw[k / 64, n] * 2^-F). One thread per 8 codes (4 packed bytes);
// an element whose value is not exactly a normal float16 number (or zero) is counted in *inexact.
__global__ void fold_weight_kernel(const uint8_t* __restrict__ qweight, const uint16_t* __restrict__ wscales,
                                   int scale_dtype, int N, int K, float unshift, uint16_t* __restrict__ w16,
                                   unsigned int* __restrict__ inexact) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // word index
  const int64_t words = static_cast<int64_t>(N) * K / 8;
  if (i >= words) return;
  const int64_t e0 = i * 8;
  const int n = static_cast<int>(e0 / K), k = static_cast<int>(e0 % K);
  const uint16_t sbits = wscales[static_cast<int64_t>(k / 64) * N + n];
  const float sw = scale_dtype == 1 ? __half2float(__ushort_as_half(sbits)) : __bfloat162float(__ushort_as_bfloat16(sbits));
  const float f = __fmul_rn(sw, unshift);  // exact: a power of two
  const uint32_t p = reinterpret_cast<const uint32_t*>(qweight)[i];
  uint32_t out[4];
  unsigned int bad = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t byte = (p >> (8 * j)) & 0xFFu;
    const int lo = static_cast<int>(byte << 28) >> 28, hi = static_cast<int>((byte >> 4) << 28) >> 28;
    uint32_t pair = 0;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float v = __fmul_rn(static_cast<float>(t ? hi : lo), f);  // exact in float32 (<= 22 bits)
      const __half hv = __float2half_rn(v);
      const float back = __half2float(hv);
      if (back != v || (v != 0.f && fabsf(v) < 6.103515625e-05f)) ++bad;  // not exact, or a subnormal
      pair |= static_cast<uint32_t>(__half_as_ushort(hv)) << (16 * t);
    }
    out[j] = pair;
  }
  reinterpret_cast<uint4*>(w16)[i] = make_uint4(out[0], out[1], out[2], out[3]);
  if (bad) atomicAdd(inexact, bad);
}

static bool make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                        uint32_t box_inner, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace fold

int gemm_fold_validate(const GemmArgs& a, const char** why) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) {
    *why = "M, N and K must be positive";
    return 1;
  }
  if (a.N % 128 != 0 || a.N < fold::BN) {
    *why = "N must be a multiple of 128 and at least 256";
    return 1;
  }
  if (a.K % fold::BK != 0) {
    *why = "K must be a multiple of 64";
    return 1;
  }
  if (a.ep.mode == kEpiDumpGroup) {
    *why = "the folded format holds no separate integer group partials (use an E4M3 or int8 format)";
    return 1;
  }
  if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.b) | (a.lda * 2) | (a.ldb * 2)) & 15) {
    *why = "operands must be 16-byte aligned with 16-byte aligned rows";
    return 1;
  }
  if (!a.wscale || (reinterpret_cast<uintptr_t>(a.wscale) & 3)) {
    *why = "w_scales must point to the float 2^F of the folded weights";
    return 1;
  }
  return 0;
}

int gemm_fold_launch(const GemmArgs& a, cudaStream_t stream, const char** why) {
  if (gemm_fold_validate(a, why) != 0) return 1;
  CUtensorMap ma, mb;
  if (!fold::make_map_2d(&ma, a.a, a.K, a.M, a.lda * 2, fold::BK, fold::BM) ||
      !fold::make_map_2d(&mb, a.b, a.K, a.N, a.ldb * 2, fold::BK, fold::BN)) {
    *why = "cuTensorMapEncodeTiled rejected an operand (alignment or stride)";
    return 2;
  }
  const dim3 grid((a.M + fold::BM - 1) / fold::BM, (a.N + fold::BN - 1) / fold::BN);
  cudaError_t e = cudaSuccess;
  static const bool pairs_on = [] {
    const char* v = getenv("WDL_GEMM_PAIRS");
    return !v || atoi(v) != 0;
  }();
  if (a.code_format == kCodesF16Pre && pairs_on && a.M > fold::BM) {
    // persistent CTA pairs: one pair per TPC (or per tile, when there are fewer), 2-SM MMAs on 256 x 256 tiles
    CUtensorMap mb_half;
    if (!fold::make_map_2d(&mb_half, a.b, a.K, a.N, a.ldb * 2, fold::BK, fold::BN / 2)) {
      *why = "cuTensorMapEncodeTiled rejected the weights";
      return 2;
    }
    const int tiles = ((a.M + 2 * fold::BM - 1) / (2 * fold::BM)) * ((a.N + fold::BN - 1) / fold::BN);
    auto launch_pair = [&](auto kernel) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(fold::kSmemPairBytes));
      if (e != cudaSuccess) return;
      static int resident = 0;  // pairs that fit on the GPU at once
      if (resident == 0) {
        cudaLaunchConfig_t probe = {};
        probe.gridDim = dim3(2 * 74);
        probe.blockDim = dim3(fold::kThreads);
        probe.dynamicSmemBytes = fold::kSmemPairBytes;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &probe) != cudaSuccess || clusters <= 0) {
          cudaGetLastError();  // the query is advisory: fall back to one pair per two SMs
          int dev = 0, sms = 148;
          if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
          clusters = sms / 2;
        }
        resident = clusters;
      }
      const unsigned pairs = static_cast<unsigned>(tiles < resident ? tiles : resident);
      kernel<<<dim3(2 * pairs), fold::kThreads, fold::kSmemPairBytes, stream>>>(ma, mb_half, a.wscale, a.ep, a.M, a.N,
                                                                               a.K, a.err);
    };
    switch (a.ep.mode) {
      case kEpiBf16: a.ep.lr_act ? launch_pair(fold::gemm_pre_pair_kernel<kEpiBf16, true>) : launch_pair(fold::gemm_pre_pair_kernel<kEpiBf16, false>); break;
      case kEpiResidualF32: a.ep.lr_act ? launch_pair(fold::gemm_pre_pair_kernel<kEpiResidualF32, true>) : launch_pair(fold::gemm_pre_pair_kernel<kEpiResidualF32, false>); break;
      case kEpiGeluU4: a.ep.lr_act ? launch_pair(fold::gemm_pre_pair_kernel<kEpiGeluU4, true>) : launch_pair(fold::gemm_pre_pair_kernel<kEpiGeluU4, false>); break;
      default: *why = "unknown epilogue mode"; return 1;
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
      *why = cudaGetErrorString(e);
      return 3;
    }
    return 0;
  }
  if (a.code_format == kCodesF16Pre) {  // persistent: one CTA per SM (or per tile, when there are fewer)
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tiles = static_cast<int>(grid.x * grid.y);
    const dim3 pgrid(tiles < sms ? tiles : sms);
    auto launch_p = [&](auto kernel) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(fold::kSmemPBytes));
      if (e == cudaSuccess)
        kernel<<<pgrid, fold::kThreads, fold::kSmemPBytes, stream>>>(ma, mb, a.wscale, a.ep, a.M, a.N, a.K, a.err);
    };
    switch (a.ep.mode) {
      case kEpiBf16: a.ep.lr_act ? launch_p(fold::gemm_pre_kernel<kEpiBf16, true>) : launch_p(fold::gemm_pre_kernel<kEpiBf16, false>); break;
      case kEpiResidualF32: a.ep.lr_act ? launch_p(fold::gemm_pre_kernel<kEpiResidualF32, true>) : launch_p(fold::gemm_pre_kernel<kEpiResidualF32, false>); break;
      case kEpiGeluU4: a.ep.lr_act ? launch_p(fold::gemm_pre_kernel<kEpiGeluU4, true>) : launch_p(fold::gemm_pre_kernel<kEpiGeluU4, false>); break;
      default: *why = "unknown epilogue mode"; return 1;
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
      *why = cudaGetErrorString(e);
      return 3;
    }
    return 0;
  }
  auto launch = [&](auto kernel) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(fold::kSmemBytes));
    if (e == cudaSuccess)
      kernel<<<grid, fold::kThreads, fold::kSmemBytes, stream>>>(ma, mb, a.wscale, a.ep, a.M, a.N, a.K, a.err);
  };
  switch (a.ep.mode) {
    case kEpiBf16: a.ep.lr_act ? launch(fold::gemm_fold_kernel<kEpiBf16, true>) : launch(fold::gemm_fold_kernel<kEpiBf16, false>); break;
    case kEpiResidualF32: a.ep.lr_act ? launch(fold::gemm_fold_kernel<kEpiResidualF32, true>) : launch(fold::gemm_fold_kernel<kEpiResidualF32, false>); break;
    case kEpiGeluU4: a.ep.lr_act ? launch(fold::gemm_fold_kernel<kEpiGeluU4, true>) : launch(fold::gemm_fold_kernel<kEpiGeluU4, false>); break;
    default: *why = "unknown epilogue mode"; return 1;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return 3;
  }
  return 0;
}

void fold_weight_launch(const uint8_t* qweight, const uint16_t* wscales, int scale_dtype, int N, int K, int shift,
                        uint16_t* w16, unsigned int* inexact, cudaStream_t stream) {
  const int64_t words = static_cast<int64_t>(N) * K / 8;
  fold::fold_weight_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, stream>>>(
      qweight, wscales, scale_dtype, N, K, ldexpf(1.f, -shift), w16, inexact);
}

}  // namespace w4a4
}  // namespace wdl
