"""Oracle of SageAttention over the FP8 KV cache. Test infrastructure only (see oracle/__init__.py).

Reference (src/wan_dit_lab/kernels/sage_kv.py; SageAttention 2.2.0's kernel itself is third-party and absent):
  - _load :29-40 — tokens [0, at) are cache FP8 x per-(token, head) scale, [at, at + n) the chunk in float32.
  - _sum_max :44-56 — per (b, h, d) sum of K over all L tokens (mean = sum / L), and max|V|.
  - _quant_k :60-85 — K - mean to INT8: in a block of 64 tokens, scale g (0..3) covers tokens 8 i + 2 g and
    8 i + 2 g + 1; scale = max|x| / 127 + 1e-7; q = trunc(x / scale + 0.5 sign(x)) (half away from zero).
  - V_MAX = 2.25 :24; _quant_v :89-105 — v_scale[d] = max(max|V_d|, 1e-8) / 2.25, V / v_scale to E4M3,
    transposed to [B, D, H, padded tokens], permuted within 16 tokens as [0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15].
  - quant_q :112-124 — Q to INT8: within 32 tokens lane l of 8 holds tokens l, l+8, l+16, l+24 (one scale for
    the four), padded to blocks of 128; scales [B, H, blocks * 8].
  - the attention: softmax(q k^T * sq * sk * sm_scale) (v * v_scale), sm_scale = D^-0.5 (sage_kv.py:133),
    non-causal over cache and chunk (native/ops/sage_ops.cpp:15-16). Exactly computed here over the
    dequantized operands (float64); subtracting the key mean leaves softmax unchanged.
Parity unpinned for the kernel's own P V rounding (SageAttention's code is absent); the quantizers are pinned by
the reference's Triton kernels run on the CPU.

quant_v_tokens and attention_fp8_p's key_scale restate this build's own P V over the cache (not the reference's):
V stays in the cache's per-(token, head) E4M3 form, the chunk's rows quantized by the cache's own rule, and each
key's scale is folded into P before its E4M3 rounding, P = E4M3(448 p vs[t] / max vs), so that P V reads the
cache's bytes in place.
"""

import numpy as np

from oracle.fp8 import from_e4m3_bits, quantize_rows, to_e4m3_bits

V_MAX = 2.25
BLKQ, WARPQ, BLKK = 128, 32, 64
PERM16 = np.array([0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15])


def load(cache, scale, chunk, at):
    """[B, L, H, D] float32: the cache bytes times their scales before `at`, the chunk after."""
    c = from_e4m3_bits(cache[:, :at]) * np.asarray(scale[:, :at], np.float32)
    return np.concatenate([c.astype(np.float32), np.asarray(chunk, np.float32)], axis=1)


def trunc_half_away(y):
    return np.trunc(y + np.where(y >= 0, 0.5, -0.5).astype(np.float32)).astype(np.int8)


def quant_k(K):
    """K [B, L, H, D] float32 -> (k_int8 [B, L, H, D], k_scale [B, H, blocks * 4], mean [B, H, D])."""
    B, L, H, D = K.shape
    mean = (K.astype(np.float64).sum(axis=1) / L).astype(np.float32)  # [B, H, D]
    blocks = -(-L // BLKK)
    padded = np.zeros((B, blocks * BLKK, H, D), np.float32)
    padded[:, :L] = K - mean[:, None]
    x = padded.reshape(B, blocks, 8, 4, 2, H, D)  # token = 64 blk + 8 i + 2 g + j
    scale = (np.abs(x).max(axis=(2, 4, 6)) / np.float32(127.0) + np.float32(1e-7)).astype(np.float32)  # [B, blk, 4, H]
    q = trunc_half_away((x / scale[:, :, None, :, None, :, None]).astype(np.float32))
    q = q.reshape(B, blocks * BLKK, H, D)[:, :L]
    return q, scale.transpose(0, 3, 1, 2).reshape(B, H, blocks * 4), mean


def quant_v(V):
    """V [B, L, H, D] float32 -> (v_fp8 bytes [B, D, H, padded], v_scale [B, H, D])."""
    B, L, H, D = V.shape
    vmax = np.abs(V).max(axis=1)  # [B, H, D]
    v_scale = (np.maximum(vmax, np.float32(1e-8)) / np.float32(V_MAX)).astype(np.float32)
    blocks = -(-L // BLKK)
    padded = blocks * BLKK
    out = np.zeros((B, D, H, padded), np.uint8)
    q = to_e4m3_bits((V / v_scale[:, None]).astype(np.float32))  # [B, L, H, D]
    i = np.arange(L)
    j = i % 16
    pair = j // 2
    to = i - j + (pair % 4) * 4 + (pair // 4) * 2 + j % 2
    out[:, :, :, to] = q.transpose(0, 3, 2, 1)
    return out, v_scale


def quant_v_tokens(cache_v, cache_vs, V, at):
    """This build's V operand over the FP8 cache: the cached rows [0, at) as the cache holds them (E4M3 bytes and a
    scale per token and head), the chunk's rows quantized per token and head by the cache's own rule
    (oracle.fp8.quantize_rows, reference kernels/cache_fp8.py:23-41). Returns (bytes [B, L, H, D] uint8,
    scales [B, L, H] float32)."""
    c8, cs = quantize_rows(np.asarray(V, np.float32))
    codes = np.concatenate([np.asarray(cache_v[:, :at], np.uint8), c8], axis=1)
    scales = np.concatenate([np.asarray(cache_vs[:, :at], np.float32)[..., 0], cs[..., 0]], axis=1)
    return codes, scales


def unpermute_v(v_fp8, L):
    """[B, D, H, padded] Sage layout -> E4M3 bytes [B, L, H, D] in token order."""
    i = np.arange(L)
    j = i % 16
    pair = j // 2
    to = i - j + (pair % 4) * 4 + (pair // 4) * 2 + j % 2
    return v_fp8[:, :, :, to].transpose(0, 3, 2, 1)


def quant_q(Q):
    """Q [B, n, H, D] float32 -> (q_int8 [B, n, H, D], q_scale [B, H, blocks * 8])."""
    B, n, H, D = Q.shape
    blocks = -(-n // BLKQ) * (BLKQ // WARPQ)
    x = np.zeros((B, blocks * WARPQ, H, D), np.float32)
    x[:, :n] = Q
    x = x.reshape(B, blocks, 4, 8, H, D)
    scale = (np.abs(x).max(axis=(2, 5), keepdims=True) / np.float32(127.0) + np.float32(1e-7)).astype(np.float32)
    q = trunc_half_away((x / scale).astype(np.float32)).reshape(B, blocks * WARPQ, H, D)[:, :n]
    return q, scale.reshape(B, blocks, 8, H).transpose(0, 3, 1, 2).reshape(B, H, blocks * 8)


def attention(q, k, v, sm_scale=None):
    """Exact softmax(q k^T * sm_scale) v per head, float64: q [B, n, H, D], k, v [B, L, H, D]."""
    q, k, v = (np.asarray(t, np.float64) for t in (q, k, v))
    sm_scale = q.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    B, n, H, D = q.shape
    out = np.empty((B, n, H, v.shape[-1]))
    for b in range(B):
        for h in range(H):
            s = (q[b, :, h] @ k[b, :, h].T) * sm_scale
            s -= s.max(-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(-1, keepdims=True)
            out[b, :, h] = p @ v[b, :, h]
    return out


def attention_fp8_p(q, k, v_codes, v_scale, sm_scale=None, tile=128, p_scale=448.0, key_scale=None):
    """SageAttention 2's P V in FP8, per head: online softmax over key tiles of `tile` (running max m, sum l, the
    output rescaled by 2^(m_old - m_new)), each tile's P = E4M3(2^(s - m) * p_scale) times the FP8 V codes
    (float64 accumulation), the channel scale and 1 / (p_scale l) applied at the end. q, k dequantized
    [B, n, H, D] / [B, L, H, D]; v_codes [B, L, H, D] the E4M3 values of V / v_scale; v_scale [B, H, D].

    Evaluated without the loop over tiles: tile j's running max m_j is the cumulative maximum of the tiles' own
    maxima, so every tile's P (and its E4M3 rounding) is formed at once with its own m_j, and the online rescaling
    folds into one factor 2^(m_j - m_last) per tile and row. The same FP8 values as the loop; the float64 sums
    differ from it only at float64 rounding.

    key_scale [B, L, H] (v_scale then None): V's scale per key instead of per channel, folded into P before its
    E4M3 rounding as P = E4M3(p_scale 2^(s - m) key_scale[t] / max(key_scale)); the output is then
    O max(key_scale) / (p_scale l)."""
    q, k, vc = (np.asarray(t, np.float64) for t in (q, k, v_codes))
    sm_scale = q.shape[-1] ** -0.5 if sm_scale is None else sm_scale
    B, n, H, D = q.shape
    L = k.shape[1]
    out = np.empty((B, n, H, D))
    c = sm_scale * np.log2(np.e)
    tiles = -(-L // tile)
    pad = tiles * tile - L
    for b in range(B):
        for h in range(H):
            s = (q[b, :, h] @ k[b, :, h].T) * c
            st = np.pad(s, ((0, 0), (0, pad)), constant_values=-np.inf).reshape(n, tiles, tile)
            m = np.maximum.accumulate(st.max(2), axis=1)  # [n, tiles]: the running max after each tile
            p = np.exp2(st - m[:, :, None])  # each tile against its own running max
            lsum = (p.sum(2) * np.exp2(m - m[:, -1:])).sum(1)
            if key_scale is None:
                p8 = from_e4m3_bits(to_e4m3_bits((p * p_scale).astype(np.float32))).astype(np.float64)
            else:
                ks = np.asarray(key_scale[b, :, h], np.float64)
                kmax = ks.max()
                kt = np.pad(ks / kmax, (0, pad)).reshape(tiles, tile)
                p8 = from_e4m3_bits(to_e4m3_bits((p * p_scale * kt[None]).astype(np.float32))).astype(np.float64)
            p8 *= np.exp2(m - m[:, -1:])[:, :, None]  # the online rescaling, applied once per tile
            o = p8.reshape(n, tiles * tile)[:, :L] @ vc[b, :, h]
            scale = v_scale[b, h][None, :] if key_scale is None else kmax
            out[b, :, h] = o * scale / (p_scale * lsum[:, None])
    return out


def sage_attention(Q, cache_k, cache_ks, cache_v, cache_vs, at, K, V, sm_scale=None, fp8_p=False, rows=None,
                   token_v=False):
    """sage_kv.attend on the dequantized Sage operands: what the INT8 / FP8 kernel approximates, exactly; with
    fp8_p, P V in FP8 tile by tile as the kernel computes it (attention_fp8_p). rows: the query rows to compute
    (all when None); Q's INT8 scales are formed over every row first, so a row's result does not depend on which
    others are computed. token_v: this build's V over the cache (quant_v_tokens, the key scale folded into P)
    instead of the reference's per-channel V."""
    Kf = load(cache_k, cache_ks, K, at)
    kq, ks, _ = quant_k(Kf)
    qq, qs = quant_q(np.asarray(Q, np.float32))
    L = Kf.shape[1]
    kd = dequant_k(kq, ks)
    qd = dequant_q(qq, qs)
    if rows is not None:
        qd = qd[:, np.asarray(rows)]
    if token_v:
        vb, vsc = quant_v_tokens(cache_v, cache_vs, V, at)
        if fp8_p:
            return attention_fp8_p(qd, kd, from_e4m3_bits(vb), None, sm_scale, key_scale=vsc)
        return attention(qd, kd, from_e4m3_bits(vb) * vsc[..., None], sm_scale)
    v8, vs = quant_v(load(cache_v, cache_vs, V, at))
    if fp8_p:
        return attention_fp8_p(qd, kd, from_e4m3_bits(unpermute_v(v8, L)), vs, sm_scale)
    vd = from_e4m3_bits(unpermute_v(v8, L)) * vs[:, None]
    return attention(qd, kd, vd, sm_scale)


def dequant_k(kq, ks):
    B, L, H, D = kq.shape
    blocks = ks.shape[-1] // 4
    tok = np.arange(L)
    g = (tok % 8) // 2
    idx = (tok // BLKK) * 4 + g  # [L]
    scale = ks[:, :, idx].transpose(0, 2, 1)  # [B, L, H]
    return kq.astype(np.float32) * scale[..., None]


def dequant_q(qq, qs):
    B, n, H, D = qq.shape
    tok = np.arange(n)
    idx = (tok // WARPQ) * 8 + tok % 8
    scale = qs[:, :, idx].transpose(0, 2, 1)
    return qq.astype(np.float32) * scale[..., None]
