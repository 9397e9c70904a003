"""Oracle of the W4A4 (SVDQuant INT4) linear: group quantization, nibble packing, exact integer group
partials and the scaled sum. Test infrastructure only (see oracle/__init__.py).

Reference:
  - int4_groups(R, "max"): src/wan_dit_lab/quantization/w4a4.py:81-100 — scale = max(amax, 1e-8) / 7 per group
    of 64, code = round-half-even(R / scale) clamped to [-8, 7].
  - the stored scale dtype: w4a4.py:174 (bfloat16; BASELINE config 1 states float16).
  - live::w4a4_linear: native/ops/w4a4_ops.cpp:22-40 — quantize the activation per token per 64-group,
    then y = sum_g sx * sw * (int partial) + bias (Nunchaku gemm_w4a4, third-party, restated here from
    SVDQuant's published algorithm: per-group INT4 x INT4 -> INT32, promoted with both group scales).
  - smoothing: the kernel divides x by smooth before quantizing (w4a4.py:9-11, :177).
  - gelu_mlp: w4a4.py:195-204 — hidden = GELU_tanh(x W1^T + b1) + 0.171875 quantized unsigned [0, 15].
Parity unpinned for the GEMM's promotion and the unsigned hidden quantizer (Nunchaku's code is absent); the weight
and activation rounding (int4_groups) is pinned by the reference's own function.
"""

import numpy as np
import torch

GROUP = 64
GELU_SHIFT = 0.171875


def round_to(x, dtype):
    """float32 array rounded to bfloat16 / float16 (round to nearest even) and back to float32."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(getattr(torch, dtype)).float().numpy()


def int4_groups(x, smooth=None, unsigned=False):
    """Rows of x [M, K] float32 in INT4 groups of 64 (w4a4.py:86-100): codes int8 [M, K], fp32 scales [M, K/64].
    smooth [K]: x / smooth first (fp32). unsigned: codes in [0, 15] with scale = max / 15 (the hidden layer of
    gelu_mlp, whose input is GELU + 0.171875 >= 0)."""
    x = np.asarray(x, dtype=np.float32)
    if smooth is not None:
        x = (x / np.asarray(smooth, dtype=np.float32)[None, :]).astype(np.float32)
    M, K = x.shape
    g = x.reshape(M, K // GROUP, GROUP)
    top = np.maximum(np.abs(g).max(axis=-1), np.float32(1e-8))
    scale = (top / np.float32(15.0 if unsigned else 7.0)).astype(np.float32)
    q = np.rint(g / scale[..., None]).astype(np.float32)
    q = np.clip(q, 0, 15) if unsigned else np.clip(q, -8, 7)
    return q.astype(np.int8).reshape(M, K), scale


def pack_nibbles(codes):
    """codes [M, K] in [-8, 7] -> uint8 [M, K/2]: byte j holds code 2j in its low nibble, 2j+1 in its high."""
    c = np.asarray(codes).astype(np.int16) & 0xF
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed):
    """uint8 [M, K/2] -> signed codes int8 [M, K] (two's complement nibbles)."""
    p = np.asarray(packed, dtype=np.uint8).astype(np.int16)
    lo, hi = p & 0xF, p >> 4
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty((p.shape[0], p.shape[1] * 2), dtype=np.int8)
    out[:, 0::2], out[:, 1::2] = lo, hi
    return out


def group_partials(xq, wq, groups=None):
    """Exact integer group partials P[g, m, n] = sum_{k in g} xq[m, k] wq[n, k], as int32. Computed with float32
    matmuls: every term and every partial sum is an integer of magnitude < 2^24, so float32 is exact."""
    xq = np.asarray(xq, dtype=np.float32)
    wq = np.asarray(wq, dtype=np.float32)
    M, K = xq.shape
    G = K // GROUP
    groups = range(G) if groups is None else groups
    out = []
    for g in groups:
        s = slice(g * GROUP, (g + 1) * GROUP)
        out.append(xq[:, s] @ wq[:, s].T)
    return np.stack(out).astype(np.int32)


def gemm(xq, sx, wq, sw, bias=None):
    """y [M, N] float32 = sum_g sx[g, m] * sw[g, n] * P_g[m, n] + bias[n], accumulated in float32 over g in order
    (sx [K/64, M], sw [K/64, N] are the stored, rounded scales)."""
    xq = np.asarray(xq, dtype=np.float32)
    wq = np.asarray(wq, dtype=np.float32)
    sx = np.asarray(sx, dtype=np.float32)
    sw = np.asarray(sw, dtype=np.float32)
    M, K = xq.shape
    N = wq.shape[0]
    G = K // GROUP
    y = np.zeros((M, N), dtype=np.float32)
    P = np.empty((M, N), dtype=np.float32)
    S = np.empty((M, N), dtype=np.float32)
    for g in range(G):
        s = slice(g * GROUP, (g + 1) * GROUP)
        np.matmul(xq[:, s], wq[:, s].T, out=P)  # the exact integer partial P_g (float32 holds it exactly)
        np.multiply(sx[g][:, None], sw[g][None, :], out=S)  # sx * sw, exact (two bf16 / f16 values)
        np.multiply(P, S, out=P)
        np.add(y, P, out=y)  # y += P_g (sx sw), in group order
    if bias is not None:
        y += np.asarray(bias, dtype=np.float32)[None, :]
    return y


def linear(x_bf16, w_codes, w_scales, bias=None, smooth=None, scale_dtype="bfloat16"):
    """live::w4a4_linear without a low-rank branch: x [M, K] (bfloat16 values as float32) -> y float32 before the
    final bfloat16 rounding, plus the activation codes and scales it used."""
    xq, sx = int4_groups(x_bf16, smooth)
    sx_stored = round_to(sx, scale_dtype).T.copy()  # [K/64, M]
    y = gemm(xq, sx_stored, w_codes, w_scales, bias)
    return y, xq, sx_stored


def weight(W, scale_dtype="bfloat16"):
    """W [N, K] float32 -> codes [N, K] int8, fp32 scales [N, K/64], stored scales [K/64, N] (rounded)."""
    q, s = int4_groups(W)
    return q, s, round_to(s, scale_dtype).T.copy()


def gelu_tanh(x):
    x = np.asarray(x, dtype=np.float32)
    return (0.5 * x * (1.0 + np.tanh(np.float32(0.7978845608028654) * (x + np.float32(0.044715) * x ** 3)))).astype(np.float32)


def lowrank(x, down, up):
    """The SVDQuant low-rank branch (x proj_down) proj_up^T in float32: x [M, K] the layer's input before
    smoothing (proj_down is already divided by the smoothing, w4a4.py:175), down [K, r], up [N, r]
    (the bfloat16 factors as float32). Nunchaku forms it in its quantizer (lora_act, fp32) and GEMM epilogue
    (native/ops/w4a4_ops.cpp:27, 36)."""
    x = np.asarray(x, np.float32)
    return ((x @ np.asarray(down, np.float32)).astype(np.float32) @ np.asarray(up, np.float32).T).astype(np.float32)


def linear_lowrank(x_bf16, w_codes, w_scales, down, up, bias=None, smooth=None, scale_dtype="bfloat16"):
    """live::w4a4_linear with its low-rank branch: the INT4 product (linear above, no bias) + the branch + bias,
    float32 before the final bfloat16 rounding."""
    y, _, _ = linear(x_bf16, w_codes, w_scales, None, smooth, scale_dtype)
    if down is not None and np.asarray(down).size:
        y = y + lowrank(x_bf16, down, up)
    if bias is not None:
        y = y + np.asarray(bias, np.float32)[None, :]
    return y.astype(np.float32)


def gelu_mlp(x_bf16, l1, l2, scale_dtype="bfloat16"):
    """live::w4a4_gelu_mlp (w4a4_ops.cpp:44-63, w4a4.py:195-204) with low-rank branches: h = layer 1 (INT4 + branch
    + bias); g = GELU_tanh(h); the hidden layer g + 0.171875, divided by layer 2's smoothing, quantized unsigned
    (scales rounded to scale_dtype); y = layer 2's INT4 product + branch of g (without the shift) + bias. l1, l2:
    dicts codes [N, K], scales [K/64, N] (stored), down, up, bias, smooth (or None). Returns y float32."""
    h = linear_lowrank(x_bf16, l1["codes"], l1["scales"], l1["down"], l1["up"], l1["bias"], l1.get("smooth"),
                       scale_dtype)
    g = gelu_tanh(h)
    u = (g + np.float32(GELU_SHIFT)).astype(np.float32)
    hq, hs = int4_groups(u, l2.get("smooth"), unsigned=True)
    y = gemm(hq, round_to(hs, scale_dtype).T.copy(), l2["codes"], l2["scales"])
    if l2["down"] is not None and np.asarray(l2["down"]).size:
        y = y + lowrank(g, l2["down"], l2["up"])
    y = y + np.asarray(l2["bias"], np.float32)[None, :]
    return y.astype(np.float32)
