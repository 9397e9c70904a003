// The down-projection of SVDQuant's low-rank branch: act [M, rank] f32 = x [M, K] proj_down [K, rank] (Nunchaku
// forms it beside its activation quantizer, the reference's native/ops/w4a4_ops.cpp:27; the up-projection is formed
// in the GEMM epilogue, w4a4_gemm.h add_lowrank). A skinny product (rank 32 against K up to 14336) that a library
// GEMM runs far from its peak: here a cluster of S CTAs (S = 1..8, splitting K) takes 8 rows of x and 32 ranks;
// each CTA streams its slice of K through shared memory in chunks of 64 columns — its rows of x as stored and the
// 64 x 32 block of proj_down — with cp.async copies four chunks deep, so that the next chunks' loads overlap this
// chunk's arithmetic; its 8 warps split a chunk's columns, each lane accumulating one rank for the 8 rows in
// float32. The warps' partial sums are added in a fixed order, then the cluster's CTA 0 adds the CTAs' sums in rank
// order through distributed shared memory: results do not depend on timing.
#include "common.cuh"
#include "w4a4_quant.h"

#include <algorithm>

namespace wdl {
namespace w4a4 {

constexpr int kLrRows = 8, kLrChunk = 64, kLrThreads = 256, kLrStages = 4;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  // 16 bytes global -> shared, asynchronously (zero-filled when !valid: source size 0)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory"); }

template <bool kF32>
struct LrStage {
  // x rows as stored (bf16 or f32) and the chunk's block of proj_down (this CTA's 32 ranks)
  __align__(16) uint8_t x[kLrRows][kLrChunk * (kF32 ? 4 : 2)];
  __align__(16) float d[kLrChunk][32];
};

template <bool kF32>
__global__ void __launch_bounds__(kLrThreads) lowrank_down_kernel(const void* __restrict__ x, int64_t ldx, int M, int K,
                                                                  const float* __restrict__ down, int rank,
                                                                  float* __restrict__ act, int64_t ld_act) {
  constexpr int kES = kF32 ? 4 : 2;  // bytes per element of x
  __shared__ LrStage<kF32> st[kLrStages];
  static_assert(sizeof(st) >= sizeof(float) * (kLrThreads / 32) * kLrRows * 32, "the reduction reuses the stages");
  auto red = reinterpret_cast<float(*)[kLrRows][32]>(&st[0]);  // [warp][row][lane], once the stages are drained
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kLrRows;
  const int r0 = blockIdx.y * 32, r = r0 + lane;  // this CTA's ranks, this lane's rank
  // this CTA's slice of K: whole chunks, the cluster's CTAs in order
  const int split = static_cast<int>(cluster_nctas()), part = static_cast<int>(cluster_ctarank());
  const int all_chunks = (K + kLrChunk - 1) / kLrChunk;
  const int per = (all_chunks + split - 1) / split;
  const int c_begin = part * per, chunks = max(0, min(all_chunks - c_begin, per));
  // one chunk's copies: proj_down 64 rows x 32 ranks (8 x 16 bytes a row; 2 copies a thread), x 8 rows x 64
  // columns (16-byte pieces: 64 of them in bf16, 128 in f32); out-of-range pieces zero-filled
  auto issue = [&](int c) {
    LrStage<kF32>& s = st[c % kLrStages];
    const int k0 = (c_begin + c) * kLrChunk;
#pragma unroll
    for (int i = 0; i < kLrChunk * 8 / kLrThreads; ++i) {
      const int piece = threadIdx.x + i * kLrThreads;  // 0 .. 511
      const int kr = piece >> 3, q = piece & 7;        // row of the chunk, 16-byte piece of its 32 ranks
      const int k = k0 + kr, rr = r0 + q * 4;
      const bool ok = k < K && rr < rank;  // rank % 4 == 0: a piece is all in or all out
      cp_async16(&s.d[kr][q * 4], ok ? down + static_cast<int64_t>(k) * rank + rr : down, ok);
    }
    constexpr int kPieces = kLrRows * kLrChunk * kES / 16;
    for (int piece = threadIdx.x; piece < kPieces; piece += kLrThreads) {
      const int row = piece / (kLrChunk * kES / 16), col = (piece % (kLrChunk * kES / 16)) * (16 / kES);
      const int m = m0 + row, k = k0 + col;
      const bool ok = m < M && k < K;
      const uint8_t* src = static_cast<const uint8_t*>(x) + (static_cast<int64_t>(m) * ldx + k) * kES;
      cp_async16(&s.x[row][col * kES], ok ? src : x, ok);
    }
  };
  float acc[kLrRows];
#pragma unroll
  for (int i = 0; i < kLrRows; ++i) acc[i] = 0.f;
#pragma unroll
  for (int c = 0; c < kLrStages - 1; ++c) {
    if (c < chunks) issue(c);
    cp_async_commit();
  }
  for (int c = 0; c < chunks; ++c) {
    cp_async_wait<kLrStages - 2>();  // chunk c has landed (this thread's copies)
    __syncthreads();                 // everyone's copies, and everyone done with chunk c - 1's stage
    if (c + kLrStages - 1 < chunks) issue(c + kLrStages - 1);
    cp_async_commit();
    const LrStage<kF32>& s = st[c % kLrStages];
    const int kb = warp * (kLrChunk / 8);  // this warp's 8 columns of the chunk
#pragma unroll
    for (int kk = 0; kk < kLrChunk / 8; kk += 4) {
      float d[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = s.d[kb + kk + i][lane];
#pragma unroll
      for (int row = 0; row < kLrRows; ++row) {
        float xv[4];
        if constexpr (kF32) {
          const float4 v = *reinterpret_cast<const float4*>(&s.x[row][(kb + kk) * 4]);
          xv[0] = v.x, xv[1] = v.y, xv[2] = v.z, xv[3] = v.w;
        } else {
          const uint2 u = *reinterpret_cast<const uint2*>(&s.x[row][(kb + kk) * 2]);
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          xv[0] = a.x, xv[1] = a.y, xv[2] = b.x, xv[3] = b.y;
        }
        acc[row] = fmaf(xv[3], d[3], fmaf(xv[2], d[2], fmaf(xv[1], d[1], fmaf(xv[0], d[0], acc[row]))));
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp done with the stages before they hold the reduction
#pragma unroll
  for (int row = 0; row < kLrRows; ++row) red[warp][row][lane] = acc[row];
  __syncthreads();
  const int row = threadIdx.x >> 5, m = m0 + row;  // thread t sums (row t / 32, rank lane) over the warps in order
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < kLrThreads / 32; ++w) sum += red[w][row][lane];
  __syncthreads();
  float* mine = &red[0][row][lane];  // this CTA's sum, where CTA 0 of the cluster reads it
  *mine = sum;
  cluster_sync();  // every CTA's sum written (release / acquire at cluster scope)
  if (part == 0) {
    float total = sum;
    for (int p = 1; p < split; ++p) {
      float v;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(peer_smem(smem_u32(mine), p)));
      total += v;
    }
    if (m < M && r < rank) act[m * ld_act + r] = total;
  }
  cluster_sync();  // CTA 0 done reading before any CTA of the cluster exits
}

cudaError_t lowrank_down_launch(const void* x, int x_f32, int64_t ldx, int M, int K, const float* down, int rank,
                                float* act, int64_t ld_act, cudaStream_t s) {
  // K split over a cluster of up to 8 CTAs, about 512 columns each
  const int chunks = (K + kLrChunk - 1) / kLrChunk;
  const int split = std::max(1, std::min(8, chunks / 8));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((M + kLrRows - 1) / kLrRows, (rank + 31) / 32, split);
  cfg.blockDim = dim3(kLrThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = split;
  cfg.attrs = attr, cfg.numAttrs = 1;
  return x_f32 ? cudaLaunchKernelEx(&cfg, lowrank_down_kernel<true>, x, ldx, M, K, down, rank, act, ld_act)
               : cudaLaunchKernelEx(&cfg, lowrank_down_kernel<false>, x, ldx, M, K, down, rank, act, ld_act);
}

}  // namespace w4a4
}  // namespace wdl
