// SageAttention's attention on sm_100a tensor cores: O = softmax(q k^T * sq * sk * sm_scale) (v * v_scale) for
// one head and 128 queries per CTA, over all L keys (non-causal: a chunk attends to the cached frames and to
// itself, native/ops/sage_ops.cpp:15-16 of the reference), in the layouts of sage.cu.
//
// Per key tile of 128:
//   S = Q K^T               tcgen05.mma kind::i8 (int32 in TMEM), M = N = 128, K = 128
//   softmax                 4 warps, thread = query row: s = S * (q_scale * k_scale * sm_scale * log2 e),
//                           online max / sum, p = 2^(s - m); P = E4M3(p * 448) into shared memory (the 128-byte
//                           swizzled K-major layout of an MMA A operand); O rescaled in TMEM when the max grows
//   O += P V                tcgen05.mma kind::f8f6f4 (e4m3 x e4m3 -> f32 in TMEM), M = N = K = 128
// and finally O * v_scale / (448 l) in bf16. The P scale 448 and the per-channel V scale are SageAttention 2's
// FP8 P V scheme (sage_kv.py:24 V_MAX = 2.25 keeps |V / v_scale| <= 2.25).
//
// Per-token V (kTokenV, the attention over the KV cache): V stays as the FP8 cache holds it, E4M3 rows of 128
// channels with a scale vs[t] per (key, head). A tile's 128 rows arrive by TMA straight from the cache (the keys
// past rows0 from a scratch of the same layout) as the MN-major B operand of P V, and the tile's 128 scales by a
// bulk copy on the same barrier. Each key's scale is folded into P before its E4M3 rounding: with vmax the largest
// scale of the head, p' = 2^(s - m + log2 448 - log2 vmax) and P = E4M3(p' vs[t]) (<= 448), l sums p', and the
// output is O / l, no per-channel factor.
//
// Warps: 0 TMA producer (Q once, K and V tiles, 2 stages), 1 TMEM owner + MMA issuer, 2-9 softmax: warp w owns
// TMEM lanes 32 (w % 4) .. +31 (its 32 query rows) and one half of the columns, (w - 2) / 4, so that two threads
// share a row: each holds 64 scores of a tile, the pair exchanges its row maximum through shared memory (an
// mbarrier per lane quarter, two arrivals a tile, bounded waits) and keeps its own share of the row sum until the end. Four
// softmax warps per SM sub-partition hide the latency of the exponentials and the FP8 packing. TMEM: S in columns
// 0-127 (int32), O in 128-255 (fp32); 256 columns, two CTAs per SM. The next tile's Q K^T is issued before this
// tile's P V so it overlaps the softmax.
#include "common.cuh"
#include "sage.h"

#include <climits>
#include <cstdint>
#include <type_traits>

namespace wdl {
namespace sage {

constexpr int BQ = 128, BKV = 128, HD = 128;
constexpr int kAttnThreads = 320;
constexpr int kSoftmaxWarps = 8;
constexpr uint32_t kAttnTmemCols = 256;
constexpr float kPScale = 448.f;
constexpr float kLog2PScale = 8.807354922057604f;  // log2(448)

struct __align__(1024) AttnSmem {
  uint8_t q[BQ * HD];
  uint8_t k[2][BKV * HD];
  uint8_t v[2][HD * BKV];
  uint8_t p[BQ * BKV];
  float vsc[2][BKV];  // per-token V: the key scales of each stage's tile
  uint64_t q_full, kv_full[2], kv_empty[2], s_full, s_empty, p_full, o_done;
  uint64_t pair[4];  // per lane quarter: both column halves have published their values (one phase a tile)
  float row_max[2][2][BQ];  // [tile parity][column half][row]: the halves' maxima of a tile's scores
  float row_sum[2][BQ];     // [column half][row]: the halves' shares of the row sum, at the end
  uint32_t tmem_base;
};
constexpr size_t kAttnSmemBytes = sizeof(AttnSmem) + 1024;

// The int32 Q K^T sum as a float, exactly, without the conversion unit: |S| <= 128 * 127 * 127 < 2^22, so
// S + 1.5 * 2^23 is an integer in [2^23, 2^24) whose float bits are those of 0x4B400000 + S; subtracting
// 1.5 * 2^23 again is exact. An integer add and a float add instead of one conversion on the special function
// pipe, which the softmax's exponentials already keep busy (the exponent arguments skip the float add, see c').
__device__ __forceinline__ float exact_float(uint32_t s) {
  return __fsub_rn(__uint_as_float(s + 0x4B400000u), 12582912.0f);
}

// The two warps of one lane quarter (the same 32 query rows, the two column halves) exchange values through
// shared memory: each publishes its own (written before the call), arrives once on the quarter's barrier and waits
// for the phase `phase`, after which the other half's values are visible. A bounded wait (it reports code 3 and
// returns false if the other warp never arrives), so that no error path can leave a warp blocked.
__device__ __forceinline__ bool pair_exchange(uint64_t* bar, uint32_t phase, int lane, uint32_t* err) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
  return __all_sync(0xFFFFFFFFu, mbar_wait(bar, phase & 1, err, kErrWaitAccFull));
}

// kPoly: of every four exponentials of the softmax, how many are evaluated on the FMA pipe (exp2_fma) instead of
// the special function unit (ex2). Measured at 1392 queries x 5568 keys x 24 heads: 127 us with none, 133 us with
// one, 145 us with two. The softmax warps are limited by instruction issue and latency rather than by the special
// function unit (its pipe is 42 % busy), and the polynomial's nine instructions cost more issue slots than the one
// ex2 they replace; so the share is 0.
constexpr int kAttnPolyShare = 0;
template <int kPoly, bool kTokenV>
__global__ void __launch_bounds__(kAttnThreads, 2)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_v1, AttnArgs a,
                uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem& sm = *reinterpret_cast<AttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y;
  const int T = (a.L + BKV - 1) / BKV;
  const int npad = (a.nq + BQ - 1) / BQ * BQ, Lpad = T * BKV;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_empty, kSoftmaxWarps);
    mbar_init(&sm.p_full, kSoftmaxWarps);
    mbar_init(&sm.o_done, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&sm.pair[q], 2);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t t_s = tmem, t_o = tmem + BKV;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensor_map(&map_q);
      prefetch_tensor_map(&map_k);
      prefetch_tensor_map(&map_v);
      if (kTokenV) prefetch_tensor_map(&map_v1);
      const int split = (a.rows0 + BKV - 1) / BKV;  // per-token V: tiles [0, split) from the cache rows
      mbar_arrive_expect_tx(&sm.q_full, BQ * HD);
      tma_load_2d(sm.q, &map_q, &sm.q_full, 0, h * npad + qt * BQ);
      int issued = 0;
      for (int j = 0; j < T; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&sm.kv_empty[st], ((j >> 1) & 1) ^ 1, err, kErrWaitEmpty)) break;
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * BKV * HD + (kTokenV ? BKV * 4 : 0));
        tma_load_2d(sm.k[st], &map_k, &sm.kv_full[st], 0, h * Lpad + j * BKV);
        if constexpr (kTokenV) {
          if (j < split) tma_load_2d(sm.v[st], &map_v, &sm.kv_full[st], h * HD, j * BKV);
          else tma_load_2d(sm.v[st], &map_v1, &sm.kv_full[st], h * HD, j * BKV - a.rows0);
          bulk_load(sm.vsc[st], a.v_tok_scale + static_cast<int64_t>(h) * Lpad + j * BKV, BKV * 4, &sm.kv_full[st]);
        } else {
          tma_load_2d(sm.v[st], &map_v, &sm.kv_full[st], j * BKV, h * HD);
        }
        issued = j + 1;
      }
      mbar_wait(&sm.q_full, 0, err, kErrWaitFull);
      for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
        mbar_wait(&sm.kv_full[j & 1], (j >> 1) & 1, err, kErrWaitFull);
    }
  } else if (warp == 1) {
    const uint32_t id_qk = make_idesc(2, 1, 1, BQ, BKV);  // s8 x s8 -> s32
    // e4m3 x e4m3 -> f32; per-token V: B (the V rows, keys x channels) MN-major
    const uint32_t id_pv = make_idesc(1, 0, 0, BQ, HD) | (kTokenV ? 1u << 16 : 0u);
    const uint32_t q0 = smem_u32(sm.q), p0 = smem_u32(sm.p);
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.q_full, 0, err, kErrWaitFull)) &&
              __all_sync(0xFFFFFFFFu, mbar_wait(&sm.kv_full[0], 0, err, kErrWaitFull));
    if (ok) {
      tc_fence_after();
      if (elect_one()) {
        const uint32_t k0 = smem_u32(sm.k[0]);
#pragma unroll
        for (int kk = 0; kk < HD / 32; ++kk)
          mma_i8(t_s, smem_desc_k128(q0 + kk * 32), smem_desc_k128(k0 + kk * 32), id_qk, kk > 0);
        tc_commit(&sm.s_full);
      }
      __syncwarp();
    }
    for (int j = 0; j < T && ok; ++j) {
      if (j + 1 < T) {
        const int st = (j + 1) & 1;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.kv_full[st], ((j + 1) >> 1) & 1, err, kErrWaitFull)) &&
             __all_sync(0xFFFFFFFFu, mbar_wait(&sm.s_empty, j & 1, err, kErrWaitAccEmpty));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t k0 = smem_u32(sm.k[st]);
#pragma unroll
          for (int kk = 0; kk < HD / 32; ++kk)
            mma_i8(t_s, smem_desc_k128(q0 + kk * 32), smem_desc_k128(k0 + kk * 32), id_qk, kk > 0);
          tc_commit(&sm.s_full);
        }
        __syncwarp();
      }
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.p_full, j & 1, err, kErrWaitAccFull));
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t v0 = smem_u32(sm.v[j & 1]);
#pragma unroll
        for (int kk = 0; kk < BKV / 32; ++kk)
          mma_f8(t_o, smem_desc_k128(p0 + kk * 32),
                 kTokenV ? smem_desc_mn128(v0 + kk * 4096) : smem_desc_k128(v0 + kk * 32), id_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&sm.o_done);
        tc_commit(&sm.kv_empty[j & 1]);
      }
      __syncwarp();
    }
  } else {
    // ---------------- softmax: two threads per query row, 64 scores each ----------------
    const int quarter = warp & 3;      // TMEM lane quarter: the rows this warp may read
    const int half = (warp - 2) >> 2;  // column half of S, P and O
    const int row = quarter * 32 + lane;
    const int t = qt * BQ + row;  // query token
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float qs = a.q_scale[static_cast<int64_t>(h) * (npad / 32) * 8 + (t / 32) * 8 + (t % 8)];
    const float c = qs * a.sm_scale_log2;
    // per-token V: p' = 2^(s - m) 448 / vmax (P's scale and the head's largest key scale in the exponent)
    const float log2_vmax = kTokenV ? log2f(__ldg(a.v_head_max + h)) : 0.f;
    // this half's key-scale groups of a tile: columns 64 half .. + 63 hold groups 4 half .. + 3
    const float* ks_head = a.k_scale + static_cast<int64_t>(h) * (Lpad / 64) * 4 + half * 4;
    float m = -INFINITY, l = 0.f;  // l: this half's share of the row sum (of 448 p)
    bool ok = true;
    uint8_t* prow = sm.p + (row >> 3) * 1024 + (row & 7) * 128;
    float ks_next[4];  // the next tile's key scales, loaded a tile ahead (off the critical path)
#pragma unroll
    for (int i = 0; i < 4; ++i) ks_next[i] = __ldg(ks_head + i);
    for (int j = 0; j < T; ++j) {
      float w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = c * ks_next[i];
      if (j + 1 < T) {
#pragma unroll
        for (int i = 0; i < 4; ++i) ks_next[i] = __ldg(ks_head + (j + 1) * 8 + i);
      }
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.s_full, j & 1, err, kErrWaitAccFull));
      // per-token V: the tile's key scales landed with its K and V (already complete here: S was computed from
      // that K); the wait makes the bulk copy's writes visible to this warp. The stage cannot move on to tile
      // j + 2 before this tile's P is published, so the phase waited for is this tile's.
      if (kTokenV && ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.kv_full[j & 1], (j >> 1) & 1, err, kErrWaitFull));
      if (!ok) break;
      tc_fence_after();
      // This half's 64 scores are read from TMEM twice: both 32-column parts for the row maximum, then the
      // second part again once the first part's exponentials are done, so that 32 scores are held in registers,
      // not 64 (the register pressure, not the instruction count, bounds how many exponentials are in flight).
      // S is released to the next Q K^T after the second read, halfway through this tile's softmax: ample time
      // for that MMA to finish before the next tile's softmax starts.
      const uint32_t t_row = t_s + lane_off + half * 64;
      // Row max per scale group over the integer scores: w > 0 and rounding is monotonic, so max(S) * w rounds
      // to max(S * w) (the same m as scaling every score first); the two halves' maxima meet in shared memory.
      // Then one FMA per score gives the exponent argument S * w + log2(448) - m, so that 2^arg = 448 p
      // directly (P's FP8 scale folded in); l sums 448 p.
      const int lim = a.L - j * BKV - half * 64;  // valid keys of this half of the tile (all 64 but at the end)
      float alpha = 1.f, sum = 0.f;
      uint32_t pk[16];
      auto tile = [&](auto masked) {
        constexpr bool kMasked = decltype(masked)::value;
        uint32_t s[32];
        int32_t gmax[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) gmax[g] = INT32_MIN;
        {
          uint32_t s_hi[32];
          tmem_ld32(t_row, s);
          tmem_ld32(t_row + 32, s_hi);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int g = (i % 8) / 2;
            if (!kMasked || i < lim) gmax[g] = max(gmax[g], static_cast<int32_t>(s[i]));
            if (!kMasked || 32 + i < lim) gmax[g] = max(gmax[g], static_cast<int32_t>(s_hi[i]));
          }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int g = 0; g < 4; ++g)
          if (gmax[g] != INT32_MIN) mx = fmaxf(mx, exact_float(static_cast<uint32_t>(gmax[g])) * w[g]);
        sm.row_max[j & 1][half][row] = mx;
        if (!pair_exchange(&sm.pair[quarter], j, lane, err)) ok = false;
        const float m_new = fmaxf(m, fmaxf(mx, sm.row_max[j & 1][half ^ 1][row]));
        alpha = ex2(m - m_new);
        m = m_new;
        const float base = kLog2PScale - m_new - log2_vmax;
        // c' = base - 1.5 * 2^23 w (one rounding: 4e-6 of a log2 unit at most), so that fma(x, w, c') with x the
        // integer score plus 1.5 * 2^23 read as a float (exactly 1.5 * 2^23 + S, as |S| < 2^22) is S w + base:
        // an integer add and one FMA per exponent argument
        float cg[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) cg[g] = fmaf(-12582912.f, w[g], base);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          if (part == 1) {  // the second 32 scores, read again; then S is free for the next tile's Q K^T
            tmem_ld32(t_row + 32, s);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.s_empty);
          }
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const int col = part * 32 + i;
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int g = ((i + e) % 8) / 2;
              const float arg = fmaf(__uint_as_float(s[i + e] + 0x4B400000u), w[g], cg[g]);
              p[e] = e >= 4 - kPoly ? exp2_fma(arg) : ex2(arg);
              if (kMasked && col + e >= lim) p[e] = 0.f;
            }
            sum += (p[0] + p[1]) + (p[2] + p[3]);
            if constexpr (kTokenV) {  // the keys' scales, folded into P before its E4M3 rounding
              // read where it is used: a plain load would be hoisted, sixteen float4 held across the loop
              float4 v4;
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(v4.x), "=f"(v4.y), "=f"(v4.z), "=f"(v4.w)
                           : "r"(smem_u32(&sm.vsc[j & 1][half * 64 + col])));
              p[0] *= v4.x, p[1] *= v4.y, p[2] *= v4.z, p[3] *= v4.w;
            }
            const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(p[0], p[1]), __NV_SATFINITE, __NV_E4M3);
            const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(p[2], p[3]), __NV_SATFINITE, __NV_E4M3);
            pk[col / 4] = lo | (hi << 16);
          }
        }
      };
      const float m_old = m;
      if (lim >= 64) tile(std::false_type{});
      else tile(std::true_type{});
      if (!ok) break;
      l = l * alpha + sum;
      if (j > 0) {
        // P V of the previous tile must be done: O is then stable and the P buffer free
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.o_done, (j - 1) & 1, err, kErrWaitAccFull));
        if (!ok) break;
        tc_fence_after();
      }
      // P into shared memory first (its registers free), then O rescaled: both before P V of this tile is issued
#pragma unroll
      for (int chunk = 0; chunk < 4; ++chunk) {
        const int c16 = half * 4 + chunk;  // this half's 16-byte chunks of the row
        *reinterpret_cast<uint4*>(prow + ((c16 ^ (row & 7)) << 4)) =
            make_uint4(pk[chunk * 4], pk[chunk * 4 + 1], pk[chunk * 4 + 2], pk[chunk * 4 + 3]);
      }
      if (j > 0 && __any_sync(0xFFFFFFFFu, m > m_old)) {  // this half of O's columns, rescaled to the new maximum
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t o[32];
          tmem_ld32(t_o + lane_off + half * 64 + q * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_o + lane_off + half * 64 + q * 32, o);
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }
    if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&sm.o_done, (T - 1) & 1, err, kErrWaitAccFull));
    // the row sum of both halves: one more phase of the quarter's barrier after the T of the tiles
    sm.row_sum[half][row] = l;
    if (ok) ok = pair_exchange(&sm.pair[quarter], T, lane, err);
    l += sm.row_sum[half ^ 1][row];
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;  // l sums 448 p (per-token V: 448 p / vmax)
      const float* vsc = a.v_scale + h * HD;
      __nv_bfloat16* out = a.out + static_cast<int64_t>(t) * a.ld_out + h * HD;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int d0 = half * 64 + q * 32;  // this thread's 32 channels of the output row
        uint32_t o[32];
        tmem_ld32(t_o + lane_off + d0, o);
        tmem_ld_wait();
        if (t < a.nq) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int d = d0 + i + 2 * e;
              const float s0 = kTokenV ? inv : __ldg(vsc + d) * inv, s1 = kTokenV ? inv : __ldg(vsc + d + 1) * inv;
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(o[i + 2 * e]) * s0,
                                                              __uint_as_float(o[i + 2 * e + 1]) * s1);
              wv[e] = *reinterpret_cast<const uint32_t*>(&b2);
            }
            *reinterpret_cast<uint4*>(out + d0 + i) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTmemCols);
  }
}

static bool map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int attn_launch(const AttnArgs& a, uint32_t* err, cudaStream_t s, const char** why) {
  const int npad = (a.nq + BQ - 1) / BQ * BQ, Lpad = (a.L + BKV - 1) / BKV * BKV;
  CUtensorMap mq, mk, mv, mv1;
  bool ok = map_2d(&mq, a.q_i8, HD, static_cast<uint64_t>(a.H) * npad, HD) &&
            map_2d(&mk, a.k_i8, HD, static_cast<uint64_t>(a.H) * Lpad, HD);
  if (a.token_v) {
    // keys [0, rows0): the cache rows (rows past rows0 read as zero); [rows0, L): the scratch rows
    const uint64_t row1 = static_cast<uint64_t>(a.H) * HD;
    if (a.rows0 > 0) ok = ok && map_2d(&mv, a.v_rows0, a.ld_v0, a.rows0, a.ld_v0);
    if (a.rows0 < a.L) ok = ok && map_2d(&mv1, a.v_rows1, row1, a.L - a.rows0, row1);
    if (a.rows0 <= 0) mv = mv1;
    if (a.rows0 >= a.L) mv1 = mv;
  } else {
    ok = ok && map_2d(&mv, a.v_f8, Lpad, static_cast<uint64_t>(a.H) * HD, Lpad);
    mv1 = mv;
  }
  if (!ok) {
    *why = "cuTensorMapEncodeTiled rejected an attention operand";
    return 2;
  }
  auto kernel = a.token_v ? attn_kernel<kAttnPolyShare, true> : attn_kernel<kAttnPolyShare, false>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kAttnSmemBytes));
  if (e == cudaSuccess) {
    kernel<<<dim3(npad / BQ, a.H), kAttnThreads, kAttnSmemBytes, s>>>(mq, mk, mv, mv1, a, err);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    *why = cudaGetErrorString(e);
    return 3;
  }
  return 0;
}

}  // namespace sage
}  // namespace wdl
