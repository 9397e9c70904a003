"""Cross-attention's arithmetic, a design difference from the reference checked on the CPU: the reference runs
cross-attention over the prompt's 512 tokens with SDPA in bfloat16 (generation/causal.py:418-420, "sage": SDPA
only for cross-attention), this build with the Sage kernel over the prompt's keys and values quantized once per
prompt (INT8 K, FP8 V, FP8 P). The oracle's emulation of the kernel's arithmetic (oracle/sage.py, P V in FP8 tile
by tile; the kernel matches it within 5e-3 on the GPU) against exact softmax attention over the unquantized
prompt keys and values, on normalized queries and keys as RMSNorm leaves them: cosine >= 0.999 per head, the
north star's bar for attention outputs."""

import numpy as np

from oracle import sage as osage


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def test_sage_cross_attention_within_the_attention_bar_of_exact_attention():
    rng = np.random.default_rng(5)
    nq, text, H = 384, 512, 4
    scale = rng.uniform(0.7, 1.3, (1, 1, H, 128)).astype(np.float32)  # RMSNorm weights around 1
    Q = (rng.standard_normal((1, nq, H, 128)) * scale).astype(np.float32)
    K = (rng.standard_normal((1, text, H, 128)) * scale + 0.2).astype(np.float32)
    V = (rng.standard_normal((1, text, H, 128)) * 0.5).astype(np.float32)
    empty = np.zeros((1, 0, H, 128), np.uint8)
    no_scale = np.zeros((1, 0, H, 1), np.float32)
    sage = osage.sage_attention(Q, empty, no_scale, empty, no_scale, 0, K, V, fp8_p=True)
    exact = osage.attention(Q, K, V)
    per_head = [cosine(sage[:, :, h], exact[:, :, h]) for h in range(H)]
    assert min(per_head) >= 0.999, per_head
