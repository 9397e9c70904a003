/* wdl_b200.h — C ABI of the B200 (sm_100a) kernels for the Wan-5B DiT block forward of wan-dit-lab.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (cudaStream_t passed as void*),
 * launches asynchronously on that stream and returns a status: WDL_OK, or a nonzero code whose message
 * wdl_last_error() returns (per calling thread). Arguments are validated before anything is launched or
 * written; invalid arguments return WDL_ERR_ARGUMENT and touch no buffer. Outputs and scratch are allocated by
 * the caller. The functions hold no state between calls apart from the per-device error word that bounded
 * device-side waits report into (wdl_device_error).
 *
 * Dtype codes: WDL_BF16 = 0, WDL_F16 = 1, WDL_F32 = 2.
 *
 * The W4A4 GEMM entry points (wdl_w4a4_gemm*, wdl_w4a4_linear*) take their bias 16-byte aligned, like every
 * other pointer they take, and row strides (ldy, ldo, ldr, ldc, ld_add, ld_gelu, wdl_lowrank.ld_act) below 2^31
 * elements; other values return WDL_ERR_ARGUMENT.
 *
 * Each declaration names the reference interface it replaces, by file:line of the wan-dit-lab repository.
 */
#ifndef WDL_B200_H
#define WDL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WDL_OK 0
#define WDL_ERR_ARGUMENT 1 /* invalid shape, dtype, stride, alignment or bounds: nothing was launched */
#define WDL_ERR_UNSUPPORTED 2 /* valid for the reference but outside what this build implements */
#define WDL_ERR_CUDA 3 /* a CUDA runtime call failed (launch, attribute, tensor map) */
#define WDL_ERR_DEVICE 4 /* a kernel reported a device-side error (see wdl_device_error) */

#define WDL_BF16 0
#define WDL_F16 1
#define WDL_F32 2

/* How the W4A4 GEMM's operands hold their 4-bit integer codes, one code per byte. Both are exact for codes in
 * [-8, 15]. WDL_CODES_E4M3 holds the code's value as an FP8 E4M3 number: the
 * tensor cores (tcgen05 kind::f8f6f4) then leave float32 group partials - exact integers - that need no
 * conversion before the scale promotion. WDL_CODES_INT8 holds two's complement int8 (tcgen05 kind::i8, int32
 * partials); signed codes only. (Code 2 is not used.) */
#define WDL_CODES_INT8 0
#define WDL_CODES_E4M3 1
/* WDL_CODES_F16_FOLD holds float16 operands: activation codes as float16 integers (two bytes each), weights
 * folded with their group scales, w16 = code * sw * 2^-F (wdl_w4a4_fold_weight), exact when the weight scales are
 * bf16. The GEMM (tcgen05 kind::f16) then accumulates sw * 2^-F * P per group exactly and its epilogue needs one
 * fused multiply-add by sx * 2^F per element and group; results equal WDL_CODES_E4M3's bit for bit. In this
 * format the GEMM's w_scales argument points to the single float 2^F, activation scales are [K/64, M] f32 as in
 * WDL_CODES_E4M3, N % 256 == 0, K % 64 == 0, and the group-partials view is not available. */
#define WDL_CODES_F16_FOLD 3
/* WDL_CODES_F16_PRE: float16 activations with their bf16 group scales folded in as well, float16(code * sx *
 * 2^-E_m) with one power of two per row m (8 times the row's largest |value| in [2^14, 2^15)), and the rows'
 * 2^E_m [M] float32 as the activation "scales"; weights as WDL_CODES_F16_FOLD (the same folded buffers). Both
 * operands then carry every scale: the GEMM accumulates all of K on the tensor cores (no per-group promotion) and
 * multiplies each row by 2^E_m 2^F once. Exact operands (a code has <= 3 significant bits, a bf16 scale 8; a group
 * whose scale is below 2^-25 of its row's largest rounds to float16 subnormals, and one that then loses bits is
 * reported as device error 8, see wdl_device_error); the sum is the tensor core's
 * float32 accumulation, within float32 rounding of the per-group promotion (not bit-identical to it). Written by
 * wdl_w4a4_quantize_rows / wdl_ln_quant (bf16 scales only); signed codes only: the GELU epilogue of a GEMM in
 * this format writes the (unsigned) hidden layer in WDL_CODES_F16_FOLD. The default of the Python layer. */
#define WDL_CODES_F16_PRE 4

/* Message of the last failed call on this thread ("" if none). */
const char* wdl_last_error(void);

/* Version string of the library build. */
const char* wdl_version(void);

/* Synchronises `stream`, then reads and clears the device error word of the current device: *code = 0 when no
 * kernel recorded an error since the last call, else the first code recorded: 1-6 a bounded wait given up (the
 * kernel skipped its remaining work), 7 an index map entry out of range (read as 0), 8 a prescaled (f16pre) operand
 * that could not hold a group's values exactly (a group scale more than 2^28 below its row's largest; the values
 * were rounded: the call's result is refused). Returns WDL_OK, or WDL_ERR_DEVICE when *code != 0. No reference
 * counterpart (the reference has no device-side waits). */
int wdl_device_error(void* stream, uint32_t* code);

/* ---- W4A4 (SVDQuant INT4 weights and activations, groups of 64 input channels) --------------------------- */

/* Quantizes rows of x [M, K] (bf16 or f32, row stride ldx elements) to symmetric INT4 groups of 64 along K:
 * scale = max(max|x_g|, 1e-8) / 7 in fp32, code = round-half-even(x / scale) clamped to [-8, 7]. With smooth
 * ([K] bf16, nullable) x is divided by it first, in fp32. Writes codes [M, K] int8 (one code per byte), scales
 * [K/64, M] f32 holding the scale rounded to scale_dtype (WDL_BF16 or WDL_F16), and optionally the packed
 * nibbles [M, K/2] (byte j: low nibble = code 2j, high nibble = code 2j+1). K % 64 == 0.
 * Replaces the activation quantizer of live::w4a4_linear (native/ops/w4a4_ops.cpp:22-29) and, for rows of a
 * weight, w4a4.int4_groups(R, "max") (src/wan_dit_lab/quantization/w4a4.py:81-100). */
int wdl_w4a4_quantize_rows(const void* x, int x_dtype, int64_t ldx, const uint16_t* smooth, int M, int K,
                           int scale_dtype, int code_format, void* codes, float* scales, uint8_t* packed,
                           void* stream);

/* Unpacks a packed INT4 weight: qweight [N, K/2] (low nibble = even k, two's complement) and wscales [K/64, N]
 * (scale_dtype WDL_BF16 or WDL_F16) into codes [N, K] (one byte each, code_format) and scales [K/64, N] f32,
 * the device layout of wdl_w4a4_gemm. The load-time counterpart of the packing in w4a4.quantize
 * (src/wan_dit_lab/quantization/w4a4.py:171-179). */
int wdl_w4a4_unpack_weight(const uint8_t* qweight, const void* wscales, int scale_dtype, int N, int K,
                           int code_format, void* codes, float* scales, void* stream);

/* Folds a packed INT4 weight (qweight [N, K/2], wscales [K/64, N] bf16 or f16) into float16 operands of
 * WDL_CODES_F16_FOLD: w16 [N, K] = code * wscale * 2^-shift. Adds to *inexact (a device counter the caller zeroes)
 * the number of elements that are not exactly a normal float16 number; with any, the layer must use another code
 * format. bf16 scales and shift = ceil(log2(8 * max wscale)) - 15 make every element exact unless the layer's group
 * scales span more than about 2^25. The load-time counterpart of w4a4.quantize (w4a4.py:171-179) for this format. */
int wdl_w4a4_fold_weight(const uint8_t* qweight, const void* wscales, int scale_dtype, int N, int K, int shift,
                         uint16_t* w16, uint32_t* inexact, void* stream);

/* y [M, N] bf16 (row stride ldy) = sum_g a_scales[g, m] * w_scales[g, n] * (sum_{k in g} a[m, k] w[n, k]) + bias[n]
 * on tcgen05 tensor cores. a [M, K] and w [N, K] codes in code_format (activation codes [-8, 15], weight codes
 * [-8, 7]), scales f32 ([K/64, M] and [K/64, N]), bias f32 [N] nullable. N % 256 == 0, K % 128 == 0, 16-byte
 * aligned pointers. The GEMM of live::w4a4_linear (native/ops/w4a4_ops.cpp:36-38). */
int wdl_w4a4_gemm(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                  const float* bias, int M, int N, int K, uint16_t* y, int64_t ldy, void* stream);

/* Same product, fused with the gated residual update of a Wan block:
 * out [M, N] f32 = residual[m, n] + float(bf16(product + bias[n])) * gate[n]   (gate nullable: factor 1).
 * out may alias residual. The residual additions of WanBlock.forward (src/wan_dit_lab/models/block.py:76-79). */
int wdl_w4a4_gemm_residual(const void* a, const float* a_scales, const void* w, const float* w_scales,
                           int code_format, const float* bias, const float* gate, const float* residual, int64_t ldr,
                           int M, int N, int K, float* out, int64_t ldo, void* stream);

/* Debug / parity view of the same GEMM: out [M, N] int32 (row stride ldo) = the exact integer partial
 * sum_{k in group} a[m, k] w[n, k] of one group of 64 input channels, read from the tensor-core accumulator
 * (TMEM) as the promotion sees it. No reference counterpart (Nunchaku keeps these in registers); it pins the
 * integer accumulators bit for bit. */
int wdl_w4a4_gemm_group_partials(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                 int code_format, int M, int N, int K, int group, int32_t* out, int64_t ldo,
                                 void* stream);

/* The first layer of the fused feed forward (Nunchaku's fused_gelu_mlp, live::w4a4_gelu_mlp of
 * native/ops/w4a4_ops.cpp:44-63; quantization/w4a4.py:195-204): the same product plus bias, then
 * u = GELU_tanh(y) + shift (shift 0.171875 = GELU_SHIFT makes u >= 0), divided by the next layer's smoothing
 * smooth_next ([N] bf16, nullable), quantized to UNSIGNED INT4 per group of 64 outputs (scale = max(max u, 1e-8)
 * / 15, code = round-half-even(u / scale) in [0, 15]) straight into the next layer's operand: codes [M, ldc]
 * (E4M3 format) and scales [N / 64, M] f32 rounded to scale_dtype. The hidden layer never exists in 16 bits.
 * code_format must be WDL_CODES_E4M3 or one of the float16 formats. */
int wdl_w4a4_gemm_gelu_u4(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                          const float* bias, const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N,
                          int K, uint8_t* codes, int64_t ldc, float* scales, void* stream);

/* The same three GEMMs with the SVDQuant low-rank branch: `addend` [M, ld_add] f32 (nullable) is added to the
 * product before the bias, i.e. lora_act * proj_up^T with lora_act = x * proj_down (w4a4_ops.cpp:27, 36: Nunchaku
 * computes both in the activation quantizer and the GEMM epilogue; here the caller forms the rank-r products, plain
 * GEMMs, and the epilogue adds them before the bf16 rounding, residual update or GELU). The GELU variant can also
 * write gelu_out [M, ld_gelu] f32 = GELU(y) before shift and smoothing: the input of the next layer's low-rank
 * branch (w4a4.py:195-204, the branch reads the hidden activation without the shift). */
int wdl_w4a4_gemm_add(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                      const float* bias, const float* addend, int64_t ld_add, int M, int N, int K, uint16_t* y,
                      int64_t ldy, void* stream);
int wdl_w4a4_gemm_residual_add(const void* a, const float* a_scales, const void* w, const float* w_scales,
                               int code_format, const float* bias, const float* addend, int64_t ld_add,
                               const float* gate, const float* residual, int64_t ldr, int M, int N, int K, float* out,
                               int64_t ldo, void* stream);
int wdl_w4a4_gemm_gelu_u4_add(const void* a, const float* a_scales, const void* w, const float* w_scales,
                              int code_format, const float* bias, const float* addend, int64_t ld_add,
                              const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N, int K,
                              uint8_t* codes, int64_t ldc, float* scales, float* gelu_out, int64_t ld_gelu,
                              void* stream);

/* An SVDQuant low-rank branch formed inside the GEMM epilogue (Nunchaku adds lora_act proj_up^T in its GEMM,
 * native/ops/w4a4_ops.cpp:31-40): act [M, ld_act] f32 = x proj_down (the layer's input times its down-projection,
 * computed by the caller), up [N, rank] f32 = proj_up, rank a multiple of 4 (<= 1024); every epilogue thread adds
 * act[m, :] . up[n, :] to its products before the bias, so the [M, N] product is never written to memory. act and
 * up 16-byte aligned, ld_act a multiple of 4. */
typedef struct wdl_lowrank {
  const float* act;
  int64_t ld_act;
  const float* up;
  int rank;
} wdl_lowrank;

/* The branch's down-projection: act [M, ld_act] f32 = x [M, ldx] (x_dtype WDL_BF16 or WDL_F32) proj_down [K, rank]
 * f32 (row-major, rank columns), accumulated in float32 in a fixed order (Nunchaku forms it beside its activation
 * quantizer, native/ops/w4a4_ops.cpp:27). K a multiple of 32, rank a positive multiple of 4, x and its rows
 * 16-byte aligned, proj_down 16-byte aligned, ld_act >= rank. */
int wdl_lowrank_down(const void* x, int x_dtype, int64_t ldx, int M, int K, const float* down, int rank, float* act,
                     int64_t ld_act, void* stream);

/* The _add entry points above with the branch given as a wdl_lowrank (null: none) instead of its addend. */
int wdl_w4a4_gemm_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                          const float* bias, const wdl_lowrank* lowrank, int M, int N, int K, uint16_t* y,
                          int64_t ldy, void* stream);
int wdl_w4a4_gemm_residual_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                   int code_format, const float* bias, const wdl_lowrank* lowrank, const float* gate,
                                   const float* residual, int64_t ldr, int M, int N, int K, float* out, int64_t ldo,
                                   void* stream);
int wdl_w4a4_gemm_gelu_u4_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales,
                                  int code_format, const float* bias, const wdl_lowrank* lowrank,
                                  const uint16_t* smooth_next, float shift, int scale_dtype, int M, int N, int K,
                                  uint8_t* codes, int64_t ldc, float* scales, float* gelu_out, int64_t ld_gelu,
                                  void* stream);

/* out [M, ldo] f32 = the GEMM's product (+ addend, + bias when given), not rounded: a tensor-parallel shard's
 * share of a row-parallel layer (its slice of the K input channels), summed across shards (NCCL all-reduce) before
 * wdl_residual_update applies bias, bf16 rounding, gate and residual. Groups of 64 never straddle shards, so each
 * shard's INT4 activation groups are those of the whole layer. No reference counterpart (the reference runs one
 * GPU per stream); the row-parallel split of O, cross-O and FFN-2 that this serves is described with the
 * reference's linears (quantization/w4a4.py:220-262). */
int wdl_w4a4_gemm_f32(const void* a, const float* a_scales, const void* w, const float* w_scales, int code_format,
                      const float* bias, const float* addend, int64_t ld_add, int M, int N, int K, float* out,
                      int64_t ldo, void* stream);
int wdl_w4a4_gemm_f32_lowrank(const void* a, const float* a_scales, const void* w, const float* w_scales,
                              int code_format, const float* bias, const wdl_lowrank* lowrank, int M, int N, int K,
                              float* out, int64_t ldo, void* stream);

/* Bytes of scratch wdl_w4a4_linear needs for M tokens of K channels (any code format). */
size_t wdl_w4a4_linear_workspace(int M, int K);

/* y [M, N] bf16 = x W^T + bias for x [M, K] bf16 (row stride ldx): activation quantization (smooth nullable)
 * then the W4A4 GEMM, W given as unpacked codes [N, K] (code_format) and scales [K/64, N] f32. workspace:
 * caller-owned device scratch of wdl_w4a4_linear_workspace(M, K) bytes, 256-byte aligned. live::w4a4_linear
 * (native/ops/w4a4_ops.cpp:31-40), without the low-rank branch (proj_down / proj_up of rank 0). */
int wdl_w4a4_linear(const uint16_t* x, int64_t ldx, int M, int K, const uint16_t* smooth, int scale_dtype,
                    const void* w, const float* w_scales, int code_format, const float* bias, int N, uint16_t* y,
                    int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* The W4A4 linear of wdl_w4a4_linear for callers that cannot allocate device memory: no workspace argument and
 * no allocation of any kind inside. Its scratch (the activation's INT4 codes and scales between the quantizer and
 * the GEMM) is a fixed array of WDL_W4A4_LINEAR_NOALLOC_MAX_BYTES in the library's own device memory, held by
 * every device that loads the library until the process exits. Calls needing more than that (M * K * 17 / 16
 * bytes, rounded up) return WDL_ERR_ARGUMENT. The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress) and should come before any stream capture. All calls on a device share the array: calls
 * that overlap on the GPU race and must be ordered by the caller. code_format WDL_CODES_INT8 or WDL_CODES_E4M3;
 * otherwise as wdl_w4a4_linear: a call it refuses launches nothing and leaves the array as it was.
 * No counterpart in the reference: live::w4a4_linear always allocates its scratch (native/ops/w4a4_ops.cpp:22-29). */
#define WDL_W4A4_LINEAR_NOALLOC_MAX_BYTES ((size_t)16 << 20)
int wdl_w4a4_linear_noalloc(const uint16_t* x, int64_t ldx, int M, int K, const uint16_t* smooth, int scale_dtype,
                            const void* w, const float* w_scales, int code_format, const float* bias, int N, uint16_t* y,
                            int64_t ldy, void* stream);

/* ---- 3D RoPE, the FP8 KV cache, the QKV preparation of self-attention ------------------------------------- */

/* Stores K and V [B, N, H, D] (dtypes WDL_BF16 / WDL_F16 / WDL_F32, element strides k_strides[4], v_strides[4],
 * any positive strides) into rows [at, at + N) of the FP8 caches cache_k, cache_v [B, capacity, H, D] (E4M3,
 * contiguous) with one float32 scale per (token, head) in cache_ks, cache_vs [B, capacity, H]:
 * scale = max(max|x|, 1e-12) / 448, byte = round-to-nearest-even(x / scale). Nothing else is written.
 * kernels/cache_fp8.py:75-105 store_kv_fp8 (arithmetic of quantization/fp8.py:37-41 quantize_rows). */
int wdl_store_kv_fp8(const void* k, int k_dtype, const int64_t* k_strides, const void* v, int v_dtype,
                     const int64_t* v_strides, int B, int N, int H, int D, uint8_t* cache_k, float* cache_ks,
                     uint8_t* cache_v, float* cache_vs, int capacity, int at, void* stream);

/* Rotates x [B, L, H, D] (dtype 0 bf16, 1 f16, 2 f32, 3 f64; element strides x_strides[4]) by 3D RoPE into out
 * [B, L, H, D] (contiguous, out_dtype). grids [B, 3] host array of (frames, height, width) per sample (B <= 64);
 * freq [2, positions, D/2] (f32 or f64, element strides freq_strides[3]) the cos / sin table; start: time
 * position of the first frame. Computed in float32, or float64 when x or freq is float64; tokens past
 * f h w copied. kernels/rope_triton.py:101-144 rope_apply (forward), models/rope.py:12-31. */
int wdl_rope_apply(const void* x, int x_dtype, const int64_t* x_strides, int B, int L, int H, int D, const int* grids,
                   const void* freq, int freq_dtype, const int64_t* freq_strides, int positions, int start, void* out,
                   int out_dtype, void* stream);

/* The QKV chain of self-attention on a chunk of n tokens, from one read of each row of qkv [n, ld] bf16
 * (q | k | v, dim = heads x 128 channels each, dim in {1024, 2048, 3072, 4096}): RMSNorm of q and of k over all
 * dim channels (float32 statistics, rounded to bf16, times the float32 weights norm_q / norm_k), 3D RoPE of both
 * with the float32 table freq [2, positions, 64] (chunk grid (n / (grid_h grid_w), grid_h, grid_w), time
 * position start for its first frame), q_out / k_out [n, dim] float32, and, when cache_k is not null, the rotated
 * K and the raw V stored into the FP8 cache rows [at, at + n) of cache_k / cache_v [capacity, heads, 128] with
 * their per-(token, head) scales. FusedQKVAttention.forward (quantization/w4a4.py:252-262) with
 * MultiHeadAttention's norms (models/multi_head_attention.py:28-44) and KVCache.store
 * (generation/causal.py:177-184). */
int wdl_qkv_prep(const uint16_t* qkv, int64_t ld, int n, int dim, const float* norm_q, const float* norm_k, float eps,
                 const float* freq, int positions, int grid_h, int grid_w, int start, float* q_out, float* k_out,
                 uint8_t* cache_k, float* cache_ks, uint8_t* cache_v, float* cache_vs, int capacity, int at,
                 void* stream);

/* wdl_qkv_prep on a tensor-parallel shard's heads: dim = this shard's heads x 128 (any multiple of 128 up to
 * 4096), norm_q / norm_k its slices of the weights, and sumsq [n, 2] f32 the sums of squares of each token's q and
 * k over all norm_dim channels of all shards (wdl_rows_sumsq per shard, summed across shards), so that the RMSNorm
 * divides by the whole row's statistics. sumsq null: the shard is the whole row (norm_dim must equal dim). The
 * cache rows hold this shard's heads ([capacity, dim / 128, 128]). MultiHeadAttention's q / k norms span all heads
 * (models/multi_head_attention.py:28-44). */
int wdl_qkv_prep_sharded(const uint16_t* qkv, int64_t ld, int n, int dim, const float* norm_q, const float* norm_k,
                         float eps, const float* sumsq, int norm_dim, const float* freq, int positions, int grid_h,
                         int grid_w, int start, float* q_out, float* k_out, uint8_t* cache_k, float* cache_ks,
                         uint8_t* cache_v, float* cache_vs, int capacity, int at, void* stream);

/* ---- normalizations of the block, fused with what consumes them ------------------------------------------- */

/* LayerNorm of x [M, K] (x_dtype WDL_F32 or WDL_BF16, row stride ldx; K % 256 == 0, K <= 4096) over K channels
 * (float32 statistics, eps; ln_w / ln_b [K] float32 affine, nullable), rounded to bf16 when round_ln_bf16 (the
 * residual stream is bf16: .type_as), then when mod_shift is not null y * (1 + mod_scale) + mod_shift (float32
 * [K] each), then rounded to bf16 (the next linear layer's input) and quantized as wdl_w4a4_quantize_rows does
 * (smooth [K] bf16 nullable): codes [M, K] (code_format), scales [K / 64, M] (scale_dtype). The [K] vectors are
 * 16-byte aligned.
 * models/block.py:75-79 norm1 / norm2 (modulated) and norm3 (affine) feeding quantization/w4a4.py:229-231. */
int wdl_ln_quant(const void* x, int x_dtype, int64_t ldx, int M, int K, float eps, const float* ln_w,
                 const float* ln_b, int round_ln_bf16, const float* mod_shift, const float* mod_scale,
                 const uint16_t* smooth, int scale_dtype, int code_format, void* codes, float* scales, void* stream);
/* wdl_ln_quant that also writes the layer's bf16 input (after LayerNorm and modulation, before the smoothing)
 * to x_out [M, ld_xo]: what an SVDQuant low-rank branch multiplies by proj_down (Nunchaku's activation quantizer
 * forms x proj_down from the same values, native/ops/w4a4_ops.cpp:27). */
int wdl_ln_quant_keep(const void* x, int x_dtype, int64_t ldx, int M, int K, float eps, const float* ln_w,
                      const float* ln_b, int round_ln_bf16, const float* mod_shift, const float* mod_scale,
                      const uint16_t* smooth, int scale_dtype, int code_format, void* codes, float* scales,
                      uint16_t* x_out, int64_t ld_xo, void* stream);

/* RMSNorm of rows: out [M, ldo] f32 = bf16(x * rsqrt(mean(x^2) + eps)) * w for x [M, ldx] bf16 (K % 256 == 0,
 * K <= 4096; x, w and out 16-byte aligned). models/rms_norm.py:10-13 (the query norm of cross-attention, models/multi_head_attention.py:118). */
int wdl_rms_rows(const uint16_t* x, int64_t ldx, int M, int K, const float* w, float eps, float* out, int64_t ldo,
                 void* stream);

/* wdl_rms_rows over a shard's slice of K channels (K % 128 == 0) of rows normalized over norm_dim channels:
 * sumsq [M] f32 holds each row's sum of squares over all of them (nullable: the slice is the row, norm_dim = K). */
int wdl_rms_rows_sharded(const uint16_t* x, int64_t ldx, int M, int K, const float* w, float eps, const float* sumsq,
                         int norm_dim, float* out, int64_t ldo, void* stream);

/* out [M, parts] f32: the sum of squares of each bf16 row's `parts` slices of K channels (slice p starts at
 * channel p * part_stride; K % 8 == 0, 16-byte aligned rows). A shard's share of an RMSNorm's statistics. */
int wdl_rows_sumsq(const uint16_t* x, int64_t ldx, int M, int K, int parts, int64_t part_stride, float* out,
                   void* stream);

/* x [M, ldx] f32 += gate * float(bf16(partial + bias)) (gate, bias [N] f32 nullable: gate 1, bias 0), for
 * partial [M, ldp] f32 the all-reduced product of a row-parallel layer: the residual epilogue of
 * wdl_w4a4_gemm_residual after the sum across shards (models/block.py:76-79 X + y * gate). N % 4 == 0. */
int wdl_residual_update(const float* partial, int64_t ldp, const float* bias, const float* gate, float* x, int64_t ldx,
                        int M, int N, void* stream);

/* out [blocks, 6, dim] f32 = time_in [6, dim] + modulation [blocks, 6, dim]: the (time_in + self.modulation)
 * of every block of a model at once (models/block.py:75). */
int wdl_modulation(const float* time_in, const float* modulation, int blocks, int dim, float* out, void* stream);

/* ---- SageAttention over the FP8 KV cache ----------------------------------------------------------------- */
/* Layouts of the quantized operands (this library's own; SageAttention's sm89 layouts are kernel-internal):
 *   q_i8 [H, npad, 128] int8, q_scale [H, npad / 32 * 8] f32      token t: scale (t / 32) * 8 + t % 8
 *   k_i8 [H, Lpad, 128] int8, k_scale [H, Lpad / 64 * 4] f32      key j:   scale (j / 64) * 4 + (j % 8) / 2
 *   v_f8 [H, 128, Lpad] e4m3 (keys contiguous), v_scale [H, 128] f32
 * npad = nq rounded up to 128, Lpad = L = at + n rounded up to 128; padding holds zero codes.
 * Cache: cache_k / cache_v [capacity, H, 128] e4m3 with scales cache_ks / cache_vs [capacity, H] (batch 1).
 * Chunk: k [n, ld_k], v [n, ld_v] (k_dtype / v_dtype WDL_F32 or WDL_BF16), head h at column h * 128.
 * Alignment: cache bases 4 bytes; chunk bases 16 bytes (float32) or 8 bytes (bf16) with ld_k, ld_v multiples of
 * 4; q 16 bytes with ld_q a multiple of 4; q_i8, k_i8, v_f8 and v_scale 16 bytes. */

/* The quantization of SageAttention 2 read straight from the FP8 cache (tokens [0, at)) and the chunk
 * (tokens [at, at + n)): key mean over all L = at + n keys, K - mean to INT8 with 4 scales per 64 keys
 * (keys 8 i + 2 g, 8 i + 2 g + 1; scale max|x| / 127 + 1e-7, round half away from zero), V / v_scale to E4M3
 * with v_scale = max(max|V_d|, 1e-8) / 2.25 per channel, Q [nq, ld_q] float32 to INT8 with one scale per
 * 4 tokens (l, l + 8, l + 16, l + 24 of 32). work: wdl_sage_prep_workspace(L, H) bytes of scratch.
 * kernels/sage_kv.py:29-124 (_load, _sum_max, _quant_k, _quant_v, quant_q). */
size_t wdl_sage_prep_workspace(int L, int H);
int wdl_sage_prep(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                  const uint8_t* cache_v, const float* cache_vs, int at, const void* k, int k_dtype, int64_t ld_k,
                  const void* v, int v_dtype, int64_t ld_v, int n, int H, int8_t* q_i8, float* q_scale, int8_t* k_i8,
                  float* k_scale, uint8_t* v_f8, float* v_scale, void* work, size_t work_bytes, void* stream);

/* out [nq, ld_out] bf16 (head h at column h * 128) = softmax(q k^T * q_scale * k_scale * sm_scale) (v * v_scale)
 * over all L keys, non-causal, from the quantized operands above: INT8 Q K^T on tcgen05 kind::i8, P = E4M3(448 p)
 * times FP8 V on kind::f8f6f4, fp32 accumulation in TMEM. live::sage_sm89 (native/ops/sage_ops.cpp:12-19). */
int wdl_sage_attention(const int8_t* q_i8, const float* q_scale, const int8_t* k_i8, const float* k_scale,
                       const uint8_t* v_f8, const float* v_scale, int nq, int L, int H, float sm_scale, uint16_t* out,
                       int64_t ld_out, void* stream);

/* The K / V half of wdl_sage_prep alone (the keys and values of cross-attention are quantized once per prompt:
 * at = 0, the prompt's n tokens as the chunk), and the Q half alone. */
int wdl_sage_prep_kv(const uint8_t* cache_k, const float* cache_ks, const uint8_t* cache_v, const float* cache_vs,
                     int at, const void* k, int k_dtype, int64_t ld_k, const void* v, int v_dtype, int64_t ld_v, int n,
                     int H, int8_t* k_i8, float* k_scale, uint8_t* v_f8, float* v_scale, void* work, size_t work_bytes,
                     void* stream);
int wdl_sage_quant_q(const float* q, int64_t ld_q, int nq, int H, int8_t* q_i8, float* q_scale, void* stream);

/* Attention over the FP8 KV cache in one call: sage_kv.attend (kernels/sage_kv.py:127-176) with heads = tokens =
 * None, scratch in the caller's workspace of wdl_sage_attend_workspace(nq, L, H) bytes (256-byte aligned). Q and
 * K are quantized as wdl_sage_prep does. V is not re-quantized per channel: P V reads V as the cache holds it,
 * E4M3 rows with a scale per (token, head), through TMA in place (cache_v 16-byte aligned), each key's scale
 * folded into P before its E4M3 rounding (P = E4M3(448 p vs[t] / max vs), out = O / sum(448 p / max vs)). The
 * chunk's values v are quantized per (token, head) by the cache's own rule (kernels/cache_fp8.py:23-41) into the
 * workspace; v = null means the caller has already stored them in the cache at rows [at, at + n) (wdl_qkv_prep
 * does), so that every key is read from the cache. */
size_t wdl_sage_attend_workspace(int nq, int L, int H);
int wdl_sage_attend(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                    const uint8_t* cache_v, const float* cache_vs, int at, const void* k, int k_dtype, int64_t ld_k,
                    const void* v, int v_dtype, int64_t ld_v, int n, int H, float sm_scale, uint16_t* out,
                    int64_t ld_out, void* workspace, size_t workspace_bytes, void* stream);

/* wdl_sage_attend with Forcing-KV's index maps (sage_kv.attend heads / tokens, kernels/sage_kv.py:127-134; used by
 * KVCache.attend_split, generation/causal.py:222-240): the cache holds cache_rows rows of cache_heads heads
 * ([cache_rows, cache_heads, 128] and [cache_rows, cache_heads]); head h of the call (of q, k, v, out; H of them)
 * is cache head heads[h] (null: h, and then cache_heads == H); cached key j < at is cache row tokens[j] (null: row
 * j, and then at <= cache_rows). Neither copies the cache's keys; its values are gathered through the maps into
 * the workspace in their E4M3 form (v may not be null here). A map entry out of range is read as 0 and reported in
 * the device error word (wdl_device_error). */
int wdl_sage_attend_maps(const float* q, int64_t ld_q, int nq, const uint8_t* cache_k, const float* cache_ks,
                         const uint8_t* cache_v, const float* cache_vs, int cache_rows, int cache_heads,
                         const int32_t* heads, const int32_t* tokens, int at, const void* k, int k_dtype, int64_t ld_k,
                         const void* v, int v_dtype, int64_t ld_v, int n, int H, float sm_scale, uint16_t* out,
                         int64_t ld_out, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WDL_B200_H */
