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
// with npad, Lpad multiples of 128 and zero codes in the padding. wdl_sage_attend instead keeps V as the cache
// holds it (token_v): E4M3 rows with a scale per (token, head), read in place by the attention kernel's TMA, the
// keys past rows0 in a scratch of the same row layout, and the scales gathered per head into v_tok_scale
// [H][Lpad] (see v_token_tile).
#include "common.cuh"
#include "sage.h"

namespace wdl {
namespace sage {

__device__ __forceinline__ uint8_t e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// Channels d .. d + 3 (d % 4 == 0) of token j of head h, as _load of sage_kv.py:29-40 reads them: the cache
// bytes times their scale before `at`, the chunk's values after. One 32-bit load of four E4M3 bytes (decoded two
// at a time through f16x2, exactly), or one 16-byte / 8-byte load of four float32 / bf16 values.
// With Forcing-KV's maps (sage_kv.py:127-134): head h of the call is cache head hmap[h] (the cache keeping all
// cache_H of them) and cached key j is cache row tmap[j]; an entry out of range is reported (kErrIndex) and read
// as row / head 0. Without maps, key j is row j and head h is cache head h.
struct Source {
  const uint8_t* cache;  // [cache_rows, cache_H, 128]
  const float* scale;    // [cache_rows, cache_H]
  const void* chunk;     // [n, ld] float32 (keys) or bf16 (values), head h at column h * 128
  int64_t ld;
  int chunk_bf16;
  int at, L, H;
  int cache_H, cache_rows;
  const int* hmap;  // [H] or null
  const int* tmap;  // [at] or null
  uint32_t* err;
  __device__ __forceinline__ int cache_head(int h) const {
    if (!hmap) return h;
    const int c = __ldg(hmap + h);
    if (c < 0 || c >= cache_H) {
      atomicCAS(err, 0u, static_cast<uint32_t>(kErrIndex));
      return 0;
    }
    return c;
  }
  __device__ __forceinline__ int64_t cache_row(int j) const {
    if (!tmap) return j;
    const int r = __ldg(tmap + j);
    if (r < 0 || r >= cache_rows) {
      atomicCAS(err, 0u, static_cast<uint32_t>(kErrIndex));
      return 0;
    }
    return r;
  }
  __device__ __forceinline__ void get4(int j, int h, int d, float (&o)[4]) const {
    if (j < at) {
      const int64_t r = cache_row(j) * cache_H + cache_head(h);
      const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(cache + r * 128 + d));
      const float s = __ldg(scale + r);
      const __half2 lo(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xFFFFu), __NV_E4M3));
      const __half2 hi(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3));
      const float2 a = __half22float2(lo), b = __half22float2(hi);
      o[0] = a.x * s, o[1] = a.y * s, o[2] = b.x * s, o[3] = b.y * s;
      return;
    }
    const int64_t off = static_cast<int64_t>(j - at) * ld + h * 128 + d;
    if (chunk_bf16) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(chunk) + off));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      o[0] = a.x, o[1] = a.y, o[2] = b.x, o[3] = b.y;
    } else {
      const float4 f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(chunk) + off));
      o[0] = f.x, o[1] = f.y, o[2] = f.z, o[3] = f.w;
    }
  }

  // Channels d .. d + 3 of N keys j[0..N) (those with valid[i]), all loads issued before any is used. `where`:
  // 1 every key is in the cache, 2 every key in the chunk, 0 mixed (then key by key through get4).
  template <int N>
  __device__ __forceinline__ void gather4(const int (&j)[N], const bool (&valid)[N], int where, int h, int d,
                                          float (&o)[N][4]) const {
    if (where == 1) {
      uint32_t w[N];
      float s[N];
      int64_t rows[N];
      const int ch = cache_head(h);
#pragma unroll
      for (int i = 0; i < N; ++i) rows[i] = valid[i] ? cache_row(j[i]) : 0;  // all map loads before the data loads
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int64_t r = rows[i] * cache_H + ch;
        w[i] = valid[i] ? __ldg(reinterpret_cast<const uint32_t*>(cache + r * 128 + d)) : 0u;
        s[i] = valid[i] ? __ldg(scale + r) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const __half2 lo(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] & 0xFFFFu), __NV_E4M3));
        const __half2 hi(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[i] >> 16), __NV_E4M3));
        const float2 a = __half22float2(lo), b = __half22float2(hi);
        o[i][0] = a.x * s[i], o[i][1] = a.y * s[i], o[i][2] = b.x * s[i], o[i][3] = b.y * s[i];
      }
    } else if (where == 2 && chunk_bf16) {
      uint2 u[N];
#pragma unroll
      for (int i = 0; i < N; ++i)
        u[i] = valid[i] ? __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(chunk) +
                                                               static_cast<int64_t>(j[i] - at) * ld + h * 128 + d))
                        : make_uint2(0u, 0u);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i].x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i].y));
        o[i][0] = a.x, o[i][1] = a.y, o[i][2] = b.x, o[i][3] = b.y;
      }
    } else if (where == 2) {
      float4 f[N];
#pragma unroll
      for (int i = 0; i < N; ++i)
        f[i] = valid[i] ? __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(chunk) +
                                                                static_cast<int64_t>(j[i] - at) * ld + h * 128 + d))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < N; ++i) o[i][0] = f[i].x, o[i][1] = f[i].y, o[i][2] = f[i].z, o[i][3] = f[i].w;
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (valid[i]) get4(j[i], h, d, o[i]);
        else o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      }
    }
  }
  // where the keys [j0, j1) lie: 1 all cached, 2 all in the chunk, 0 both
  __device__ __forceinline__ int where(int j0, int j1) const { return j1 <= at ? 1 : (j0 >= at ? 2 : 0); }
};

// ---- pass 1: per (64-token tile, head), per channel: sum of K (blockIdx.z 0) or max |V| (blockIdx.z 1) over the
// tile. Warp w reads the 16 tokens 16 w .. 16 w + 15 of the tile, lane l channels 4 l .. 4 l + 3 (one 128-byte row
// segment per token), all 16 of its loads in flight; the four warps' partials meet in shared memory. K and V in
// separate CTAs: each has one round of loads to wait for, and twice as many CTAs hide each other's latency.
// Per-token V of the attention over the cache (PrepArgs::token_v).
struct VTok {
  int on, rows0, Lpad;
  uint8_t* rows;       // scratch rows [rows0, L), pitch H * 128 bytes
  float* tok_scale;    // [H][Lpad]
  float* tile_max;     // [tiles][H]: each 64-key tile's largest scale
};

// Per-token V, per (64-key tile, head): each key's scale (a cached key's from the cache; a chunk key's
// max(max|v|, 1e-12) / 448 over its 128 channels, the cache's own rule, reference kernels/cache_fp8.py:23-41), into
// v_tok_scale; the keys from rows0 on written to the scratch rows (a cached key's bytes as the cache holds them, a
// chunk key's as E4M3(v / scale), the division correctly rounded); the tile's largest scale into tile_max. Keys
// past L get scale 0. Warp w holds keys 16 w .. 16 w + 15 in four rounds of four; lanes 8 i .. 8 i + 7 share one
// key, 16 channels each (the key's maximum over its eight lanes by shuffles within the group).
__device__ __forceinline__ void v_token_tile(const Source& vs, const VTok& vt, int tile, int h, float (&red)[4][128]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 3, seg = lane & 7;
  const unsigned group = 0xFFu << (sub * 8);
  float top = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = tile * 64 + warp * 16 + r * 4 + sub;
    float sc = 0.f;
    if (t < vs.L) {
      uint4 bytes = make_uint4(0u, 0u, 0u, 0u);
      if (t < vs.at) {
        const int64_t row = vs.cache_row(t) * vs.cache_H + vs.cache_head(h);
        sc = __ldg(vs.scale + row);
        if (t >= vt.rows0) bytes = __ldg(reinterpret_cast<const uint4*>(vs.cache + row * 128 + seg * 16));
      } else {
        float x[16];
        const int64_t off = static_cast<int64_t>(t - vs.at) * vs.ld + h * 128 + seg * 16;
        if (vs.chunk_bf16) {
          const uint2* p = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(vs.chunk) + off);
          uint2 u[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) u[i] = __ldg(p + i);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i].x));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i].y));
            x[4 * i] = a.x, x[4 * i + 1] = a.y, x[4 * i + 2] = b.x, x[4 * i + 3] = b.y;
          }
        } else {
          const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(vs.chunk) + off);
          float4 f[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) f[i] = __ldg(p + i);
#pragma unroll
          for (int i = 0; i < 4; ++i) x[4 * i] = f[i].x, x[4 * i + 1] = f[i].y, x[4 * i + 2] = f[i].z, x[4 * i + 3] = f[i].w;
        }
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(group, amax, o));
        sc = __fdiv_rn(fmaxf(amax, 1e-12f), 448.f);
        const float rcp = __frcp_rn(sc);
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i / 4] |= static_cast<uint32_t>(e4m3(div_rn_by(x[i], sc, rcp))) << (8 * (i % 4));
        bytes = make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (t >= vt.rows0)
        *reinterpret_cast<uint4*>(vt.rows + static_cast<int64_t>(t - vt.rows0) * vs.H * 128 + h * 128 + seg * 16) = bytes;
    }
    if (seg == 0) vt.tok_scale[static_cast<int64_t>(h) * vt.Lpad + t] = sc;
    top = fmaxf(top, sc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
  if (lane == 0) red[0][warp] = top;
  __syncthreads();
  if (threadIdx.x == 0) vt.tile_max[static_cast<int64_t>(tile) * vs.H + h] = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
}

// Per channel d of head h over the keys of the 64-key tile: their sum (kMax false) or largest |x| (kMax true), into
// out[d] by thread d. Warp w takes keys 16 w .. 16 w + 15. Cached keys (FP8): lane (sub, seg) = (lane / 8, lane % 8)
// reads the 16 bytes of channels 16 seg .. + 15 of keys 16 w + 4 r + sub (r = 0..3), one 16-byte load each, and
// folds them in as they are dequantized; chunk or mixed keys: lane l channels 4 l .. + 3 of the 16 keys in two
// batches of 8. The CTA then combines its 16 partials per channel (warp-major, sub-group-minor, a fixed order).
// Few registers a thread, so that many CTAs are resident (at 95 registers five were, and the grid ran in seven
// waves of long-scoreboard stalls).
template <bool kMax>
__device__ __forceinline__ void tile_reduce(const Source& src, int tile, int h, float (&red)[4][4][128], float* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j0 = tile * 64 + warp * 16;
  const int where = src.where(j0, min(src.L, j0 + 16));
  if (where == 1) {
    const int sub = lane >> 3, seg = lane & 7;
    const int ch = src.cache_head(h);
    uint4 w[4];
    float sc[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int j = j0 + 4 * r + sub;
      const bool ok = j < src.L;
      const int64_t row = (ok ? src.cache_row(j) : 0) * src.cache_H + ch;
      w[r] = ok ? __ldg(reinterpret_cast<const uint4*>(src.cache + row * 128 + seg * 16)) : make_uint4(0u, 0u, 0u, 0u);
      sc[r] = ok ? __ldg(src.scale + row) : 0.f;
    }
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t u[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 lo(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(u[q] & 0xFFFFu), __NV_E4M3));
        const __half2 hi(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(u[q] >> 16), __NV_E4M3));
        const float2 a = __half22float2(lo), b = __half22float2(hi);
        const float x[4] = {a.x * sc[r], a.y * sc[r], b.x * sc[r], b.y * sc[r]};
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[4 * q + c] = kMax ? fmaxf(acc[4 * q + c], fabsf(x[c])) : acc[4 * q + c] + x[c];
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) red[warp][sub][seg * 16 + i] = acc[i];
  } else {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      int j[8];
      bool valid[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) j[i] = j0 + 8 * half + i, valid[i] = j[i] < src.L;
      float x[8][4];
      src.gather4(j, valid, src.where(j[0], min(src.L, j[0] + 8)), h, lane * 4, x);
#pragma unroll
      for (int i = 0; i < 8; ++i)  // keys in order
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c] = kMax ? fmaxf(acc[c], fabsf(x[i][c])) : acc[c] + x[i][c];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      red[warp][0][lane * 4 + c] = acc[c];
      red[warp][1][lane * 4 + c] = red[warp][2][lane * 4 + c] = red[warp][3][lane * 4 + c] = 0.f;
    }
  }
  __syncthreads();
  const int d = threadIdx.x;
  float r = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int sub = 0; sub < 4; ++sub) r = kMax ? fmaxf(r, red[w][sub][d]) : r + red[w][sub][d];
  out[d] = r;
}

__global__ void __launch_bounds__(128, 8) partials_kernel(Source ks, Source vs, float* ksum, float* vmax, VTok vt) {
  __shared__ float red[4][4][128];
  const int tile = blockIdx.x, h = blockIdx.y;
  const bool is_v = blockIdx.z != 0;
  if (is_v && vt.on) {  // the grid spans Lpad / 64 tiles: the scales of the padding keys are written as 0
    v_token_tile(vs, vt, tile, h, red[0]);
    return;
  }
  if (tile * 64 >= ks.L) return;
  const int64_t o = (static_cast<int64_t>(tile) * ks.H + h) * 128;
  if (is_v) tile_reduce<true>(vs, tile, h, red, vmax + o);
  else tile_reduce<false>(ks, tile, h, red, ksum + o);
}

// ---- pass 2: per head: key mean (sum / L) and the V channel scales max(max|V|, 1e-8) / 2.25 (V_MAX, :24). CTA
// (h, c) holds channels 32 c .. 32 c + 31; its warp w sums tiles w, w + 4, ... (16 loads in flight), and the four
// warps' sums are added in a fixed order: a short dependent chain instead of one thread walking every tile.
// With per-token V (vtile_max set), vmax and v_scale are unused and CTA (h, 0) also takes the largest of head h's
// tile maxima into v_head_max[h].
__global__ void __launch_bounds__(128) reduce_kernel(const float* ksum, const float* vmax, int tiles, int H, int L,
                                                     float* kmean, float* v_scale, const float* vtile_max,
                                                     int vtiles, float* v_head_max) {
  __shared__ float red[2][4][32];
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = blockIdx.y * 32 + lane;
  if (vtile_max) {
    if (blockIdx.y == 0) {
      float top = 0.f;
      for (int t = threadIdx.x; t < vtiles; t += 128) top = fmaxf(top, vtile_max[static_cast<int64_t>(t) * H + h]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
      if (lane == 0) red[1][warp][0] = top;
    }
    float s = 0.f;
    int t = warp;
    for (; t + 28 < tiles; t += 32) {
      float a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = ksum[(static_cast<int64_t>(t + 4 * i) * H + h) * 128 + d];
#pragma unroll
      for (int i = 0; i < 8; ++i) s += a[i];
    }
    for (; t < tiles; t += 4) s += ksum[(static_cast<int64_t>(t) * H + h) * 128 + d];
    red[0][warp][lane] = s;
    __syncthreads();
    if (warp == 0) {
      const float sum = (red[0][0][lane] + red[0][1][lane]) + (red[0][2][lane] + red[0][3][lane]);
      kmean[h * 128 + d] = __fdiv_rn(sum, static_cast<float>(L));
      if (blockIdx.y == 0 && lane == 0)  // floored: a head whose every scale is 0 keeps log2(vmax) finite
        v_head_max[h] = fmaxf(fmaxf(fmaxf(red[1][0][0], red[1][1][0]), fmaxf(red[1][2][0], red[1][3][0])), 1e-30f);
    }
    return;
  }
  float s = 0.f, m = 0.f;
  int t = warp;
  for (; t + 28 < tiles; t += 32) {
    float a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] = ksum[(static_cast<int64_t>(t + 4 * i) * H + h) * 128 + d];
      b[i] = vmax[(static_cast<int64_t>(t + 4 * i) * H + h) * 128 + d];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) s += a[i], m = fmaxf(m, b[i]);
  }
  for (; t < tiles; t += 4) {
    s += ksum[(static_cast<int64_t>(t) * H + h) * 128 + d];
    m = fmaxf(m, vmax[(static_cast<int64_t>(t) * H + h) * 128 + d]);
  }
  red[0][warp][lane] = s, red[1][warp][lane] = m;
  __syncthreads();
  if (warp == 0) {
    const float sum = (red[0][0][lane] + red[0][1][lane]) + (red[0][2][lane] + red[0][3][lane]);
    const float top = fmaxf(fmaxf(red[1][0][lane], red[1][1][lane]), fmaxf(red[1][2][lane], red[1][3][lane]));
    kmean[h * 128 + d] = __fdiv_rn(sum, static_cast<float>(L));
    v_scale[h * 128 + d] = __fdiv_rn(fmaxf(top, 1e-8f), 2.25f);
  }
}

// Sage's INT8 rounding: trunc(y + 0.5 sign(y)) with y = x / scale (the division correctly rounded).
__device__ __forceinline__ uint32_t sage_i8(float x, float scale, float rcp) {
  const float y = div_rn_by(x, scale, rcp);
  return static_cast<uint32_t>(static_cast<int>(truncf(__fadd_rn(y, y >= 0.f ? 0.5f : -0.5f)))) & 0xFFu;
}

// ---- pass 3: K - mean to INT8 (kV false) or V to FP8 (kV true), per (64-key block, head). 128 threads.
// K (_quant_k, sage_kv.py:60-85): warp g holds the 16 keys 8 i + 2 g, 8 i + 2 g + 1 (i = 0..7) of the block;
// scale = max|x| / 127 + 1e-7 over the 16 x 128 values; code = trunc(x / scale + 0.5 sign(x)).
// V (_quant_v, :89-105): warp g keys 16 g .. 16 g + 15, lane l channels 4 l .. 4 l + 3, each
// V / v_scale[d] rounded to E4M3; the codes are transposed through shared memory (each lane packs its 16 keys
// of a channel into one 16-byte store) and leave as one 64-byte row segment per channel.
constexpr int kVtPitch = 80;  // bytes per channel row of the transpose tile: 16-byte aligned, reads conflict-free

template <bool kV>
__global__ void __launch_bounds__(128) quant_kv_kernel(Source ks, Source vs, const float* kmean, const float* v_scale,
                                                       int Lpad, int8_t* k_i8, float* k_scale, uint8_t* v_f8) {
  __shared__ __align__(16) uint8_t vt[kV ? 128 * kVtPitch : 16];
  const int blk = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = ks.L;
  if constexpr (!kV) {
    const int g = warp;
    const float4 mean = *reinterpret_cast<const float4*>(kmean + h * 128 + lane * 4);
    float x[16][4];
    float amax = 0.f;
    int jj[16];
    bool valid[16];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) jj[2 * i + e] = blk * 64 + 8 * i + 2 * g + e, valid[2 * i + e] = jj[2 * i + e] < L;
    ks.gather4(jj, valid, ks.where(blk * 64, min(L, blk * 64 + 64)), h, lane * 4, x);
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float* r = x[t];
      if (valid[t]) {
        r[0] = __fsub_rn(r[0], mean.x), r[1] = __fsub_rn(r[1], mean.y);
        r[2] = __fsub_rn(r[2], mean.z), r[3] = __fsub_rn(r[3], mean.w);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) amax = fmaxf(amax, fabsf(r[c]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
    const float rcp = __frcp_rn(scale);
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = blk * 64 + 8 * i + 2 * g + e;
        uint32_t packed = 0;
        if (j < L)
#pragma unroll
          for (int c = 0; c < 4; ++c) packed |= sage_i8(x[2 * i + e][c], scale, rcp) << (8 * c);
        *reinterpret_cast<uint32_t*>(k_i8 + (static_cast<int64_t>(h) * Lpad + j) * 128 + lane * 4) = packed;
      }
    if (lane == 0) k_scale[static_cast<int64_t>(h) * (Lpad / 64) * 4 + blk * 4 + g] = scale;
  } else {
    const int g = warp;
    const float4 sv = *reinterpret_cast<const float4*>(v_scale + h * 128 + lane * 4);
    const float s[4] = {sv.x, sv.y, sv.z, sv.w};
    float rcp[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) rcp[c] = __frcp_rn(s[c]);
    uint32_t w[4][4];  // [channel c][key word]: keys 16 g + 4 kw .. + 3 of channel 4 lane + c
    int jj[16];
    bool valid[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) jj[t] = blk * 64 + g * 16 + t, valid[t] = jj[t] < L;
    float v[16][4];
    vs.gather4(jj, valid, vs.where(blk * 64, min(L, blk * 64 + 64)), h, lane * 4, v);
#pragma unroll
    for (int kw = 0; kw < 4; ++kw) {
#pragma unroll
      for (int c = 0; c < 4; ++c) w[c][kw] = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b)
        if (valid[kw * 4 + b])
#pragma unroll
          for (int c = 0; c < 4; ++c)
            w[c][kw] |= static_cast<uint32_t>(e4m3(div_rn_by(v[kw * 4 + b][c], s[c], rcp[c]))) << (8 * b);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(vt + (lane * 4 + c) * kVtPitch + g * 16) = make_uint4(w[c][0], w[c][1], w[c][2], w[c][3]);
    __syncthreads();
    const int d = threadIdx.x;
    const uint4* src = reinterpret_cast<const uint4*>(vt + d * kVtPitch);
    uint4* dst = reinterpret_cast<uint4*>(v_f8 + (static_cast<int64_t>(h) * 128 + d) * Lpad + blk * 64);
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = src[q];
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
    if (t < n) {
      const float4* src = reinterpret_cast<const float4*>(q + static_cast<int64_t>(t) * ldq + h * 128 + c * 8);
      const float4 a = __ldg(src), b = __ldg(src + 1);
      x[r][0] = a.x, x[r][1] = a.y, x[r][2] = a.z, x[r][3] = a.w;
      x[r][4] = b.x, x[r][5] = b.y, x[r][6] = b.z, x[r][7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[r][i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[r][i]));
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const float scale = __fadd_rn(__fdiv_rn(amax, 127.f), 1e-7f);
  const float rcp = __frcp_rn(scale);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = blk * 32 + r * 8 + l;
    uint32_t w[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i / 4] |= sage_i8(x[r][i], scale, rcp) << (8 * (i % 4));
    *reinterpret_cast<uint2*>(q_i8 + (static_cast<int64_t>(h) * npad + t) * 128 + c * 8) = make_uint2(w[0], w[1]);
  }
  if (c == 0) q_scale[static_cast<int64_t>(h) * (npad / 32) * 8 + blk * 8 + l] = scale;
}

void prep_kv_launch(const PrepArgs& a, cudaStream_t s) {
  const int L = a.at + a.n;
  const int cache_H = a.cache_H > 0 ? a.cache_H : a.H;
  Source ks{a.cache_k, a.cache_ks, a.k_chunk, a.ld_k, a.k_bf16, a.at, L, a.H, cache_H, a.cache_rows, a.hmap, a.tmap,
            a.err};
  // no chunk values (per-token V only): the chunk's rows are in the cache already, every key is a cached one
  Source vs{a.cache_v, a.cache_vs, a.v_chunk, a.ld_v, a.v_bf16, a.v_chunk ? a.at : L, L, a.H, cache_H, a.cache_rows,
            a.hmap, a.tmap, a.err};
  const int tiles = (L + 63) / 64;
  const int Lpad = (L + 127) / 128 * 128;
  float* ksum = a.work;
  float* vmax = ksum + static_cast<int64_t>(tiles) * a.H * 128;  // per-token V: the tile maxima [Lpad / 64][H]
  float* kmean = vmax + static_cast<int64_t>(tiles) * a.H * 128;
  const VTok vt{a.token_v, a.rows0, Lpad, a.v_rows, a.v_tok_scale, vmax};
  partials_kernel<<<dim3(a.token_v ? Lpad / 64 : tiles, a.H, 2), 128, 0, s>>>(ks, vs, ksum, vmax, vt);
  reduce_kernel<<<dim3(a.H, 4), 128, 0, s>>>(ksum, vmax, tiles, a.H, L, kmean, a.v_scale, a.token_v ? vmax : nullptr,
                                             Lpad / 64, a.v_head_max);
  quant_kv_kernel<false><<<dim3(Lpad / 64, a.H), 128, 0, s>>>(ks, vs, kmean, a.v_scale, Lpad, a.k_i8, a.k_scale, a.v_f8);
  if (!a.token_v)  // V per channel, in its own kernel (its registers would hold the K kernel to fewer CTAs)
    quant_kv_kernel<true><<<dim3(Lpad / 64, a.H), 128, 0, s>>>(ks, vs, kmean, a.v_scale, Lpad, a.k_i8, a.k_scale, a.v_f8);
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
