"""Oracle of Wan's 3D RoPE, RMSNorm and LayerNorm. Test infrastructure only (see oracle/__init__.py).

Reference:
  - rope(pos_count, pos_dim): src/wan_dit_lab/models/rope.py:4-10 — cos/sin of positions * 10000^(-2i/dim)
    in float64, stacked [2, positions, dim / 2].
  - the table of a head of d = 128: pairs split 22 / 21 / 21 over time / height / width
    (models/rope.py:16-17; runtime/live_presets.py:52-61 builds it with dims d - 4 (d // 6), 2 (d // 6), 2 (d // 6)).
  - rope_apply(X, grid, freq, start_frame): models/rope.py:12-31 — token t of a (f, h, w) grid has positions
    (start_frame + t // (h w), t // w % h, t % w); x1' = x1 c - x2 s, x2' = x2 c + x1 s in the table's dtype
    (float32 in Live, runtime/live_presets.py:34), cast back to X's dtype. Tokens past f h w are copied unchanged
    (the Triton variant, kernels/rope_triton.py:54-56).
  - RMSNorm: models/rms_norm.py:10-13; LayerNorm: models/layer_norm.py:5-7 (statistics in float32).
"""

import numpy as np
import torch


def rope(count, dim):
    positions = np.arange(count, dtype=np.float64)[:, None]
    frequencies = 10000.0 ** (-2 * np.arange(dim // 2, dtype=np.float64) / dim)
    angles = positions * frequencies
    return np.stack((np.cos(angles), np.sin(angles)))


def table(count, head_dim=128):
    d = head_dim
    return np.concatenate([rope(count, d - 4 * (d // 6)), rope(count, 2 * (d // 6)), rope(count, 2 * (d // 6))], axis=-1)


def split(head_dim):
    c = head_dim // 2
    return c - 2 * (c // 3), c // 3, c // 3


def angles_for(grid, freq, start, tokens):
    """(cos, sin) [tokens, pairs] of the grid's tokens, in the table's dtype."""
    f, h, w = grid
    pairs = freq.shape[-1]
    t_p, h_p, _ = split(2 * pairs)
    t = np.arange(tokens)
    pos = np.stack([start + t // (h * w), t // w % h, t % w], axis=1)
    axis = np.concatenate([np.zeros(t_p, int), np.ones(h_p, int), np.full(pairs - t_p - h_p, 2)])
    idx = pos[:, axis]  # [tokens, pairs]
    cols = np.arange(pairs)[None, :]
    return freq[0][idx, cols], freq[1][idx, cols]


def rope_apply(x, grid, freq, start=0, out_dtype=None):
    """x [B, L, H, D] float32 values; freq [2, P, D/2] (float32 or float64); returns the rotated values in the
    table's dtype, rounded to out_dtype ("bfloat16", "float32"...) when given; padding tokens copied."""
    f, h, w = grid
    n = f * h * w
    work = freq.dtype
    c, s = angles_for(grid, freq, start, n)
    c, s = c[None, :, None, :], s[None, :, None, :]
    x = np.asarray(x)
    x1 = x[:, :n, :, 0::2].astype(work)
    x2 = x[:, :n, :, 1::2].astype(work)
    out = np.array(x, dtype=work, copy=True)
    out[:, :n, :, 0::2] = x1 * c - x2 * s
    out[:, :n, :, 1::2] = x2 * c + x1 * s
    if out_dtype is not None:
        t = torch.from_numpy(np.ascontiguousarray(out))
        if work == np.float64 and out_dtype in ("bfloat16", "float16"):
            t = t.float()  # PyTorch casts float64 to 16 bits through float32
        t = t.to(getattr(torch, out_dtype))
        out = t.numpy() if out_dtype in ("float32", "float64") else t.float().numpy()  # 16-bit values as float32
    return out


def rms_norm(x, weight, eps=1e-6, round_to=None):
    """(x * rsqrt(mean(x^2) + eps)) rounded to x's dtype (round_to), then * weight (float32)."""
    x32 = np.asarray(x, dtype=np.float32)
    r = (x32 / np.sqrt((x32.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)).astype(np.float32)
    if round_to is not None:
        r = torch.from_numpy(r).to(getattr(torch, round_to)).float().numpy()
    return (r * np.asarray(weight, dtype=np.float32)).astype(np.float32)


def layer_norm(x, eps=1e-6, weight=None, bias=None):
    x = np.asarray(x, dtype=np.float64)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    y = (x - mu) / np.sqrt(var + eps)
    if weight is not None:
        y = y * weight + bias
    return y.astype(np.float32)
