// Device helpers shared by the sm_100a kernels: mbarriers, TMA tile loads, tcgen05 (TMEM allocation, MMA,
// commit, loads) and the error word every bounded wait reports into.
//
// Every spin-wait in this library is bounded. A wait that runs out writes a code into the device error word
// (wdl_device_error) and returns false; the kernel then skips its remaining work and, where it holds TMEM,
// frees it. The host reads the error word after a synchronising call (wdl_check_device_error).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

namespace wdl {

// Upper bound on the duration of one mbarrier wait, in nanoseconds of the global timer. Legitimate waits in
// these kernels last microseconds; a wait still unsatisfied after this long means a producer will never
// arrive, and the kernel gives up instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

enum DeviceError : uint32_t {
  kErrNone = 0,
  kErrWaitFull = 1,      // a consumer gave up waiting for a TMA stage
  kErrWaitEmpty = 2,     // the producer gave up waiting for a free stage
  kErrWaitAccFull = 3,   // the epilogue gave up waiting for an accumulator
  kErrWaitAccEmpty = 4,  // the MMA issuer gave up waiting for a drained accumulator
  kErrWaitScale = 5,     // the producer gave up waiting for a released scale stage
  kErrTmemAlloc = 6,     // the TMEM allocation did not return a usable address
  kErrIndex = 7,         // an index map held an entry out of range (the entry was read as 0)
  kErrInexact = 8,       // a prescaled float16 operand could not hold a group's values exactly (rounded)
};

// Two values of a prescaled operand (code * stored scale * a power of two) as float16. The conversion is exact
// unless a group's scale lies more than about 2^28 below the largest of its row (its values then fall below
// float16's resolution); `inexact` is set when any bit was lost.
__device__ __forceinline__ __half2 prescaled_pair(float v0, float v1, bool& inexact) {
  const __half2 h = __floats2half2_rn(v0, v1);
  const float2 back = __half22float2(h);
  inexact |= (back.x != v0) | (back.y != v1);
  return h;
}

// Records kErrInexact for a thread that saw an inexact prescaled value (err nullable).
__device__ __forceinline__ void report_inexact(bool inexact, uint32_t* err) {
  if (err && inexact) atomicCAS(err, 0u, static_cast<uint32_t>(kErrInexact));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------------------------
// mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %0;" ::"r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase of `bar` with the given parity to complete. Returns false (and records `code` in the
// error word) if it did not within limit_ns nanoseconds (kWaitLimitNs unless the caller passes its own, as the
// test kernel of tests/native/wait_check.cu does with a limit of about a millisecond), or if another wait has
// already given up (codes up to kErrTmemAlloc; a data error such as kErrIndex or kErrInexact stops no kernel).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      const uint32_t seen = *reinterpret_cast<volatile uint32_t*>(err);
      if (seen != 0 && seen <= kErrTmemAlloc) return false;
      if (global_ns() - start > limit_ns) {
        atomicCAS(err, 0u, code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (tiled, no multicast)
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Contiguous bytes [src, src + bytes) of global memory into shared memory (cp.async.bulk, no tensor map): both
// addresses 16-byte aligned, bytes a multiple of 16. Completes `bytes` of transaction count on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_holder, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_holder)),
               "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, 8-bit integer operands, 32-bit integer accumulator.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A * B^T with 16-bit float operands (both f16 or both bf16, per idesc) and an f32 accumulator.
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A * B^T with 8-bit float operands (types per idesc) and an f32 accumulator.
__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (shape 32x32b, 32 repetitions).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive 32-bit TMEM columns of this thread's lane written from registers (shape 32x32b, x32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads (tensor cores, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// x / s rounded to nearest even, given r = the correctly rounded reciprocal of s (__frcp_rn(s), computed once
// for many x): Markstein's method (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990): q = RN(x r), the remainder x - s q exact by one
// FMA, q' = RN(q + rem r) is the correctly rounded quotient whenever no intermediate underflows or overflows.
// Three instructions instead of a full IEEE division per element; tests check it equals __fdiv_rn.
__device__ __forceinline__ float div_rn_by(float x, float s, float r) {
  const float q = __fmul_rn(x, r);
  const float rem = __fmaf_rn(-q, s, x);
  return __fmaf_rn(rem, r, q);
}

// 2^x on the special function unit (PTX ex2.approx; -inf gives +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for the share of a softmax's exponentials taken off the special function unit (which a
// softmax over 8-bit tensor-core scores keeps the busiest unit of the SM). x is rounded to the nearest integer n by
// adding 1.5 * 2^23 (exact for |x| < 2^22: the float's last mantissa bits then hold n), f = x - n lies in
// [-0.5, 0.5], 2^f comes from a degree-4 polynomial and 2^n is added to its exponent field as the integer n << 23
// (the shift keeps n's low bits, two's complement). The polynomial was fitted to 2^f on [-0.5, 0.5] for relative
// error (Lawson's iteratively reweighted least squares on 4000 Chebyshev nodes, a near-minimax fit): 2.7e-6 at
// most in float32 Horner form (tests/test_exp2_gpu.py checks it against exp2f). x is clamped below at -100 (the
// result is then 2^-100, nothing anyone reads); arguments above 100 are not supported.
__device__ __forceinline__ float exp2_fma(float x) {
  x = fmaxf(x, -100.f);
  const float r = __fadd_rn(x, 12582912.f);
  const float f = __fsub_rn(x, __fsub_rn(r, 12582912.f));
  float p = fmaf(f, 0.009570101276040077f, 0.05591785907745361f);
  p = fmaf(p, f, 0.240247443318367f);
  p = fmaf(p, f, 0.6931217908859253f);
  p = fmaf(p, f, 0.9999992847442627f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(r) << 23));
}

// GELU in its tanh form (torch.nn.GELU(approximate="tanh"), the feed forward of models/block.py:8-9):
// 0.5 x (1 + tanh(y)), y = sqrt(2 / pi) (x + 0.044715 x^3). From tanh(y) = 1 - 2 / (e^(2y) + 1) it equals
// x - x / (e^(2y) + 1); e^(2y) = 2^(2 y log2(e)) on the special function unit, the quotient by the fast division
// (relative error of a few 1e-7, against the 2^-4 steps of the INT4 codes the result is quantized to). Saturates
// cleanly: e^(2y) -> inf gives x, e^(2y) -> 0 gives 0.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float y = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  const float e = ex2(2.885390081777927f * y);
  return x - __fdividef(x, e + 1.f);
}

// tcgen05.wait::ld that also names the 32 destination registers of the load it completes, so that the compiler
// cannot move any use of them above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored in the 128-byte swizzled layout that a TMA
// load with CU_TENSOR_MAP_SWIZZLE_128B writes: rows of 128 bytes, 8-row atoms of 1024 bytes one after another
// (stride byte offset 1024), tile base aligned to 1024 bytes. Advancing along K inside the 128-byte row is done
// by adding the byte offset to the start address.
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: one 8-row atom
  d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;                      // 128-byte swizzle
  return d;
}

// Shared-memory descriptor of an MN-major operand tile in the 128-byte swizzled layout whose MN extent is one
// 128-byte row (128 8-bit elements): rows of 128 bytes along K, 8-row atoms of 1024 bytes (what a TMA tile load
// with box {128 bytes, rows} and 128-byte swizzle writes). The stride byte offset steps from one 8-row K group to
// the next (1024 bytes); the leading byte offset, the step between 128-byte MN blocks, is never taken at this
// width (set to 16 KB).
__device__ __forceinline__ uint64_t smem_desc_mn128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(16384u >> 4) << 16;             // leading byte offset
  d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: one 8-row K group
  d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;                      // 128-byte swizzle
  return d;
}

// Instruction descriptor of a dense tcgen05.mma with both operands K-major. Bit 16 set in addition makes B
// MN-major (allowed for the 8-bit, 16-bit and tf32 formats).
//   c_format: 0 f16, 1 f32, 2 s32; a/b format: per kind (i8: 0 u8, 1 s8; f16: 0 f16, 1 bf16; f8: 0 e4m3, 1 e5m2)
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_format, uint32_t a_format, uint32_t b_format,
                                                  uint32_t m, uint32_t n) {
  return (c_format << 4) | (a_format << 7) | (b_format << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "@px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xFFFFFFFFu));
  return pred;
}

// ---------------------------------------------------------------------------------------------------------------
// CTA pairs (a cluster of two CTAs on the two SMs of a TPC): 2-SM MMAs, whose operands and accumulator are split
// between the pair. Every tcgen05 instruction of a kernel that uses them takes .cta_group::2. No multicast form is
// used: a signal the peer needs is relayed by a remote mbarrier arrive.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of the variable at this CTA's shared address `local` in the CTA of rank `rank`.
__device__ __forceinline__ uint32_t peer_smem(uint32_t local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local), "r"(rank));
  return out;
}

// Arrives once on an mbarrier of a CTA of the cluster (address from peer_smem), releasing this thread's prior
// writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// The same arrive without release semantics: a signal that hands over no write of this thread (the completion of
// tensor-core reads this thread has observed on its own barrier), so no cluster-wide fence on the way.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// The number of CTAs in this CTA's cluster.
__device__ __forceinline__ uint32_t cluster_nctas() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Every CTA of the cluster reaches this point before any goes on (all threads of all of them).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A tile into this CTA's shared memory whose completed bytes count on the mbarrier at `bar_cluster` (the pair's
// first CTA's barrier, from peer_smem(..., 0)): each CTA of a pair loads its own half of the operands and the MMA
// issuer in the first CTA waits for both halves on one barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_holder, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_holder)),
               "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

// Arrives once on this CTA's `bar` when every 2-SM tcgen05.mma this thread issued before has completed (their
// writes to both CTAs' TMEM and their reads of both CTAs' shared memory).
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A * B^T over a CTA pair, 16-bit float operands, f32 accumulator: M = 256 rows of A (128 in each
// CTA's shared memory at the same offset), N rows of B (N / 2 in each CTA), D rows 0-127 in the first CTA's TMEM
// and 128-255 in the second's. Issued by one thread of the pair's first CTA.
__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}

template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

}  // namespace wdl
