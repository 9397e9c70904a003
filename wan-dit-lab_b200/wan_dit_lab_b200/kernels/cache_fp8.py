"""FP8 (E4M3) store of keys and values into the persistent KV cache, on the B200 kernel, with the API and the
validation of the reference's src/wan_dit_lab/kernels/cache_fp8.py (store_kv_fp8, install_cache_store).

One launch quantizes K and V row by row (a row = one token of one head): scale = max(max|x|, 1e-12) / 448,
byte = round-to-nearest-even(x / scale), the arithmetic of quantization/fp8.py:37-41 quantize_rows, into
cache[:, at:at + N] and the scales into cache_ks / cache_vs [:, at:at + N, :, 0]. Inference only.
"""

import torch

from wan_dit_lab_b200 import _native


def store_kv_fp8(k, v, cache_k, cache_ks, cache_v, cache_vs, at):
    """Store [B,N,H,D] in cache[:, at:at+N] with the quantize_rows arithmetic (reference cache_fp8.py:75-105).

    Inputs may be strided. Cache buffers are contiguous and disjoint from the inputs; callers own them."""
    tensors = (k, v, cache_k, cache_ks, cache_v, cache_vs)
    if k.ndim != 4 or v.shape != k.shape or k.shape[-1] < 1:
        raise ValueError("K and V must have matching [B,N,H,D] shapes")
    if k.device.type != "cuda" or any(t.device != k.device for t in tensors):
        raise ValueError("All buffers must be on the same CUDA device")
    if any(t.requires_grad for t in tensors):
        raise ValueError("Cache store is inference-only")
    if k.dtype not in (torch.float16, torch.bfloat16, torch.float32) or v.dtype not in (
            torch.float16, torch.bfloat16, torch.float32):
        raise TypeError("K and V must be FP16, BF16 or FP32")
    if cache_k.dtype != torch.float8_e4m3fn or cache_v.dtype != cache_k.dtype:
        raise TypeError("Cache values must be FP8 E4M3FN")
    if cache_ks.dtype != torch.float32 or cache_vs.dtype != torch.float32:
        raise TypeError("Cache scales must be FP32")
    b, n, h, d = k.shape
    if cache_k.ndim != 4 or cache_k.shape != cache_v.shape or (
            cache_k.shape[0], *cache_k.shape[2:]) != (b, h, d):
        raise ValueError("Cache dimensions must match inputs")
    if cache_ks.shape != (*cache_k.shape[:3], 1) or cache_vs.shape != cache_ks.shape:
        raise ValueError("One scale is required per cache row")
    if any(not t.is_contiguous() for t in tensors[2:]):
        raise ValueError("Cache buffers must be contiguous")
    if not isinstance(at, int) or at < 0 or at + n > cache_k.shape[1]:
        raise ValueError("Write exceeds cache bounds")
    strides = lambda t: (torch.tensor(t.stride(), dtype=torch.int64))  # noqa: E731
    ks, vs = strides(k), strides(v)
    with torch.cuda.device(k.device):
        _native.check(_native.lib().wdl_store_kv_fp8(
            k.data_ptr(), _native.DTYPE_CODE[k.dtype], ks.data_ptr(), v.data_ptr(), _native.DTYPE_CODE[v.dtype],
            vs.data_ptr(), b, n, h, d, cache_k.data_ptr(), cache_ks.data_ptr(), cache_v.data_ptr(),
            cache_vs.data_ptr(), cache_k.shape[1], at, _native.stream()))


def install_cache_store(kv_cache_class):
    """Routes the FP8 path of `kv_cache_class.store` (the reference's generation.causal.KVCache, or this package's
    KVCache) through store_kv_fp8, in this process only; returns the original method for restoration
    (reference cache_fp8.py:108-121)."""
    original = kv_cache_class.store

    def store(cache, at, k, v):
        if cache.fp8:
            store_kv_fp8(k, v, cache.k, cache.ks, cache.v, cache.vs, at)
        else:
            original(cache, at, k, v)

    kv_cache_class.store = store
    return original
