"""Oracle of one Wan block forward with W4A4 linears and SageAttention over the FP8 cache. Test infrastructure
only (see oracle/__init__.py).

Reference: src/wan_dit_lab/models/block.py:22-29 (WanBlock.forward), models/multi_head_attention.py:28-44,
quantization/w4a4.py:248-262 (FusedQKVAttention), :195-204 (gelu_mlp: GELU + 0.171875, unsigned INT4 hidden),
generation/causal.py:177-220 (KVCache.store / attend with Sage), models/rope.py, models/rms_norm.py,
models/layer_norm.py. Every linear follows oracle.w4a4.linear on the packed weights given; attention is Sage's
quantization with P V in FP8 tile by tile (oracle.sage.sage_attention, fp8_p); statistics in float64. With
token_v the self-attention's P V runs over the cache's per-token V as this build computes it (oracle.sage,
token_v: V as the cache holds it, each key's scale folded into P) instead of the reference's per-channel V.
"""

import numpy as np

from oracle import fp8 as of
from oracle import rope as orope
from oracle import sage as osage
from oracle import w4a4 as ow

GELU_SHIFT = 0.171875


def bf16(x):
    return ow.round_to(np.asarray(x, np.float32), "bfloat16")


def layer(parts):
    """(codes [N, K] int8, stored scales [K/64, N] float32, bias [N] float32) of packed W4A4 parts (numpy)."""
    codes = ow.unpack_nibbles(parts["qweight"])
    return codes, parts["wscales"].astype(np.float32), parts["bias"].astype(np.float32)


def linear(x_bf16_values, parts, act_scale="bfloat16"):
    """y float32 = W4A4 linear of x (bf16 values) on the packed parts (before the bf16 rounding of the output):
    x divided by the parts' smoothing before its INT4 groups, plus the SVDQuant low-rank branch
    (x proj_down) proj_up^T when the parts have one (quantization/w4a4.py:141-180)."""
    codes, ws, b = layer(parts)
    return ow.linear_lowrank(x_bf16_values, codes, ws, parts.get("proj_down"), parts.get("proj_up"), b,
                             parts.get("smooth"), act_scale)


def layer_norm(x, eps=1e-6, w=None, b=None):
    return orope.layer_norm(x, eps, w, b)


def whole_blocks(rows, n, block=32):
    """rows (sorted query indices) as a union of whole `block`-token blocks aligned to multiples of `block` (the
    last block of the chunk may be partial): the INT8 scales of Q and of the cross-attention query are shared by
    the tokens of such a block alone (oracle.sage.quant_q), so computing only these rows gives each of them the
    values it has in the whole chunk."""
    rows = np.asarray(rows)
    starts = rows[::block]
    for i, s in enumerate(starts):
        want = np.arange(s, min(s + block, n))
        got = rows[i * block:i * block + block]
        if s % block or len(got) != len(want) or (got != want).any() or (len(want) < block and i != len(starts) - 1):
            raise ValueError("rows must be whole aligned blocks of 32 tokens (only the chunk's last may be short)")
    return rows


def block(X, mod, parts, norms, cache, at, freq, grid, start, text, heads, trace=None, rows=None, x_is_bf16=False,
          token_v=False):
    """X [n, dim] float32 (updated copy returned), mod [6, dim] float32 (time_in + modulation), parts {layer: packed
    numpy parts}, norms dict(norm_q, norm_k, cross_norm_q, cross_norm_k, norm3_w, norm3_b), cache: dict(k, ks, v, vs)
    numpy FP8 buffers [cap, H, 128] / [cap, H, 1] (written in place at `at`), text [T, dim] bf16 values (the
    prompt after the text embedding). rows (whole_blocks): finish only these query rows after the QKV projection,
    which runs over every row (the cache and the keys need all of them); returns X[rows] updated, and the trace's
    entries from "attn" on hold those rows. x_is_bf16: X is the bf16 stream entering a model's first block, whose
    first norm returns bf16 (LayerNorm's .type_as, models/layer_norm.py:5-7); the update after it is float32."""
    X = np.array(X, np.float32, copy=True)
    n, dim = X.shape
    keep = (lambda k, v: trace.__setitem__(k, np.array(v, copy=True))) if trace is not None else (lambda k, v: None)
    sh_a, sc_a, g_a, sh_f, sc_f, g_f = mod
    # self-attention
    ln1 = bf16(layer_norm(X)) if x_is_bf16 else layer_norm(X)
    x1 = bf16((ln1 * (np.float32(1) + sc_a)).astype(np.float32) + sh_a)
    keep("x1", x1)
    qkv = bf16(linear(x1, parts["self_attn.qkv"]))
    keep("qkv", qkv)
    q, k, v = qkv[:, :dim], qkv[:, dim:2 * dim], qkv[:, 2 * dim:]
    frames = n // (grid[1] * grid[2])
    rot = lambda t: orope.rope_apply(t.reshape(1, n, heads, 128), (frames, grid[1], grid[2]), freq, start)  # noqa: E731
    Q = rot(orope.rms_norm(q, norms["norm_q"], round_to="bfloat16"))
    K = rot(orope.rms_norm(k, norms["norm_k"], round_to="bfloat16"))
    V = v.reshape(1, n, heads, 128)
    cache["k"][:, at:at + n], cache["ks"][:, at:at + n] = of.quantize_rows(K)
    cache["v"][:, at:at + n], cache["vs"][:, at:at + n] = of.quantize_rows(V)
    keep("q", Q.reshape(n, dim)), keep("k", K.reshape(n, dim))
    if rows is not None:
        rows = whole_blocks(rows, n)
        X = X[rows]
    m = X.shape[0]
    A = osage.sage_attention(Q, cache["k"], cache["ks"], cache["v"], cache["vs"], at, K, V, fp8_p=True, rows=rows,
                             token_v=token_v)
    keep("attn", A.reshape(m, dim))
    o = bf16(linear(bf16(A.reshape(m, dim)), parts["self_attn.o"]))
    X = (X + o * g_a).astype(np.float32)
    keep("x_after_self", X)
    # cross-attention
    x3 = bf16(layer_norm(X, w=norms["norm3_w"], b=norms["norm3_b"]))
    keep("x3", x3)
    cq = bf16(linear(x3, parts["cross_attn.q"]))
    keep("cq", cq)
    CQ = orope.rms_norm(cq, norms["cross_norm_q"], round_to="bfloat16").reshape(1, m, heads, 128)
    T = text.shape[0]
    ck = orope.rms_norm(bf16(linear(text, parts["cross_attn.k"])), norms["cross_norm_k"], round_to="bfloat16")
    cv = bf16(linear(text, parts["cross_attn.v"]))
    keep("ck", ck), keep("cv", cv)
    empty = np.zeros((1, 0, heads, 128), np.uint8)
    CA = osage.sage_attention(CQ, empty, np.zeros((1, 0, heads, 1), np.float32), empty,
                              np.zeros((1, 0, heads, 1), np.float32), 0, ck.reshape(1, T, heads, 128),
                              cv.reshape(1, T, heads, 128), fp8_p=True)
    keep("cattn", CA.reshape(m, dim))
    co = bf16(linear(bf16(CA.reshape(m, dim)), parts["cross_attn.o"]))
    X = (X + co).astype(np.float32)
    keep("x_after_cross", X)
    # feed forward: fc1, GELU + shift quantized unsigned, fc2
    x2 = bf16((layer_norm(X) * (np.float32(1) + sc_f)).astype(np.float32) + sh_f)
    keep("x2", x2)
    f, hq, hs = feed_forward(x2, parts)
    keep("hcodes", hq), keep("hscales", hs)
    X = (X + f * g_f).astype(np.float32)
    return X


def feed_forward(x2, parts):
    """The fused GELU MLP on its bf16 input x2 (w4a4.py:195-204): (bf16 output of ffn.2 before the gate, hidden
    codes [m, ffn] int8 in [0, 15], hidden scales [ffn / 64, m] bf16-rounded)."""
    h = linear(x2, parts["ffn.0"])
    g = ow.gelu_tanh(h)
    u = (g + np.float32(GELU_SHIFT)).astype(np.float32)
    hq, hs = ow.int4_groups(u, parts["ffn.2"].get("smooth"), unsigned=True)
    hs = ow.round_to(hs, "bfloat16").T.copy()
    codes, ws, b = layer(parts["ffn.2"])
    f = ow.gemm(hq, hs, codes, ws)
    down, up = parts["ffn.2"].get("proj_down"), parts["ffn.2"].get("proj_up")
    if down is not None and np.asarray(down).size:  # the second branch reads GELU's output without the shift
        f = f + ow.lowrank(g, down, up)
    return bf16(f + b[None, :]), hq, hs
