"""Oracle of the FP8 (E4M3) KV-cache store. Test infrastructure only (see oracle/__init__.py).

Reference: quantize_rows, src/wan_dit_lab/quantization/fp8.py:37-41 (the bitwise contract of the Triton store
kernels/cache_fp8.py:23-41, tests/test_cache_fp8.py:30-44): per row (token, head) scale =
max(max|x|, 1e-12) / 448 in float32, x / scale in float32 (IEEE division), rounded to nearest-even E4M3.
"""

import numpy as np
import torch

FP8_MAX = 448.0


def to_e4m3_bits(v):
    """float32 array -> E4M3 bytes (uint8), round to nearest even, as torch's float8_e4m3fn conversion."""
    t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def from_e4m3_bits(b):
    """E4M3 bytes -> float32 values."""
    t = torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint8))
    return t.view(torch.float8_e4m3fn).float().numpy()


def quantize_rows(x):
    """x [..., d] (float32 values of any input dtype) -> (E4M3 bytes [..., d], float32 scales [..., 1])."""
    x = np.asarray(x, dtype=np.float32)
    scale = (np.maximum(np.abs(x).max(axis=-1, keepdims=True), np.float32(1e-12)) / np.float32(FP8_MAX)).astype(np.float32)
    return to_e4m3_bits(x / scale), scale


def store(cache_k, cache_ks, cache_v, cache_vs, at, k, v):
    """KVCache.store of generation/causal.py:177-184 on numpy buffers: rows [at, at + n) of the caches."""
    n = k.shape[1]
    cache_k[:, at:at + n], cache_ks[:, at:at + n] = quantize_rows(k)
    cache_v[:, at:at + n], cache_vs[:, at:at + n] = quantize_rows(v)
