"""SageAttention 2 (INT8 Q K, FP8 P V) straight over the FP8 KV cache, on the B200 kernels, with the API of the
reference's src/wan_dit_lab/kernels/sage_kv.py (attend, quant_q semantics, V_MAX).

Tokens [0, at) come from the FP8 cache (bytes times their per-(token, head) scale), [at, at + n) from the
chunk's own keys and values; the quantization is SageAttention's (key mean over all keys subtracted, K to INT8
with 4 scales per 64 keys, V to FP8 per channel with V_MAX, Q to INT8 per 4 tokens of 32), the attention runs
on tcgen05 tensor cores (libwdl_b200.so: wdl_sage_prep, wdl_sage_attention). Layout NHD, batch 1.
"""

import torch

from wan_dit_lab_b200 import _native

V_MAX = 2.25  # the largest |V| in FP8 after the channel scale (reference sage_kv.py:24)
BLKQ, WARPQ, BLKK = 128, 32, 64


def _validate(Q, cache_k, cache_ks, cache_v, cache_vs, at, K, V, heads=None, tokens=None):
    if Q.ndim != 4 or K.ndim != 4 or V.shape != K.shape:
        raise ValueError("Q, K, V must be [B, tokens, heads, head_dim] with K and V alike")
    B, nq, H, D = Q.shape
    if B != 1:
        raise ValueError("the B200 Sage path takes batch 1 (one video stream per call)")
    if D != 128 or K.shape[2] != H or K.shape[3] != D:
        raise ValueError("head_dim 128 and matching heads required")
    if (cache_k.shape[0] != 1 or cache_k.shape[3] != D or cache_v.shape != cache_k.shape
            or (heads is None and cache_k.shape[2] != H)):
        raise ValueError("Cache dimensions must match inputs")
    for name, m, count in (("heads", heads, H), ("tokens", tokens, at)):
        if m is not None and (m.dtype != torch.int32 or m.ndim != 1 or m.numel() != count or m.device != Q.device
                              or not m.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous int32 [{count}] tensor on Q's device")
    if cache_k.dtype != torch.float8_e4m3fn or cache_v.dtype != torch.float8_e4m3fn:
        raise TypeError("Cache values must be FP8 E4M3FN")
    if cache_ks.dtype != torch.float32 or cache_vs.dtype != torch.float32:
        raise TypeError("Cache scales must be FP32")
    if not isinstance(at, int) or at < 0 or (tokens is None and at > cache_k.shape[1]):
        raise ValueError("at exceeds cache bounds")
    if K.dtype not in (torch.float32, torch.bfloat16) or V.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("chunk K and V must be float32 or bfloat16")
    tensors = (Q, cache_k, cache_ks, cache_v, cache_vs, K, V)
    if any(t.device != Q.device for t in tensors) or Q.device.type != "cuda":
        raise ValueError("All tensors must be on the same CUDA device")
    if any(not t.is_contiguous() for t in (cache_k, cache_ks, cache_v, cache_vs)):
        raise ValueError("Cache buffers must be contiguous")


def _rows(x):
    """[1, n, H, D] -> [n, H * D] contiguous, keeping float32 / bf16."""
    return x[0].reshape(x.shape[1], -1).contiguous()


def prepare(Q, cache_k, cache_ks, cache_v, cache_vs, at, K, V):
    """The quantized operands SageAttention runs on, in this library's layouts (include/wdl_b200.h):
    dict(q_i8 [H, npad, 128], q_scale [H, npad / 32 * 8], k_i8 [H, Lpad, 128], k_scale [H, Lpad / 64 * 4],
    v_f8 [H, 128, Lpad] uint8 (E4M3 bytes), v_scale [H, 128])."""
    _validate(Q, cache_k, cache_ks, cache_v, cache_vs, at, K, V)
    _, nq, H, D = Q.shape
    n = K.shape[1]
    L = at + n
    npad, lpad = -(-nq // 128) * 128, -(-L // 128) * 128
    dev = Q.device
    out = dict(q_i8=torch.zeros(H, npad, 128, dtype=torch.int8, device=dev),
               q_scale=torch.zeros(H, npad // 32 * 8, device=dev),
               k_i8=torch.zeros(H, lpad, 128, dtype=torch.int8, device=dev),
               k_scale=torch.zeros(H, lpad // 64 * 4, device=dev),
               v_f8=torch.zeros(H, 128, lpad, dtype=torch.uint8, device=dev),
               v_scale=torch.zeros(H, 128, device=dev))
    q, k, v = _rows(Q.float()), _rows(K), _rows(V)
    lib = _native.lib()
    work = torch.empty(lib.wdl_sage_prep_workspace(L, H), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _native.check(lib.wdl_sage_prep(
            q.data_ptr(), q.stride(0), nq, cache_k.data_ptr(), cache_ks.data_ptr(), cache_v.data_ptr(),
            cache_vs.data_ptr(), at, k.data_ptr(), _native.DTYPE_CODE[k.dtype], k.stride(0), v.data_ptr(),
            _native.DTYPE_CODE[v.dtype], v.stride(0), n, H, *(out[name].data_ptr() for name in
                                                            ("q_i8", "q_scale", "k_i8", "k_scale", "v_f8", "v_scale")),
            work.data_ptr(), work.numel(), _native.stream()))
    return out


def attend(Q, cache_k, cache_ks, cache_v, cache_vs, at, K, V, sm_scale=None, heads=None, tokens=None):
    """softmax(Q K^T / sqrt(d)) V over the cached tokens [0, at) (FP8 cache_k, cache_v with scales per token and
    head cache_ks, cache_vs [1, tokens, H, 1]) and the chunk's own K, V [1, n, H, D]; Q [1, n_q, H, D]. Returns
    [1, n_q, H, D] in bfloat16 (reference sage_kv.py:127-134). heads (int32 [H]): head h of Q, K, V is cache head
    heads[h], the cache keeping all of them; tokens (int32 [at]): cached token i is cache token tokens[i]. Neither
    copies the cache (wdl_sage_attend_maps reads through them; an entry out of range is reported by
    wan_dit_lab_b200._native.device_error())."""
    _validate(Q, cache_k, cache_ks, cache_v, cache_vs, at, K, V, heads, tokens)
    _, nq, H, D = Q.shape
    n = K.shape[1]
    L = at + n
    sm_scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    q, k, v = _rows(Q.float()), _rows(K), _rows(V)
    out = torch.empty(1, nq, H, D, dtype=torch.bfloat16, device=Q.device)
    lib = _native.lib()
    work = torch.empty(lib.wdl_sage_attend_workspace(nq, L, H), dtype=torch.uint8, device=Q.device)
    with torch.cuda.device(Q.device):
        if heads is None and tokens is None:
            _native.check(lib.wdl_sage_attend(
                q.data_ptr(), q.stride(0), nq, cache_k.data_ptr(), cache_ks.data_ptr(), cache_v.data_ptr(),
                cache_vs.data_ptr(), at, k.data_ptr(), _native.DTYPE_CODE[k.dtype], k.stride(0), v.data_ptr(),
                _native.DTYPE_CODE[v.dtype], v.stride(0), n, H, sm_scale, out.data_ptr(), H * D, work.data_ptr(),
                work.numel(), _native.stream()))
        else:
            _native.check(lib.wdl_sage_attend_maps(
                q.data_ptr(), q.stride(0), nq, cache_k.data_ptr(), cache_ks.data_ptr(), cache_v.data_ptr(),
                cache_vs.data_ptr(), cache_k.shape[1], cache_k.shape[2], _native.ptr(heads), _native.ptr(tokens), at,
                k.data_ptr(), _native.DTYPE_CODE[k.dtype], k.stride(0), v.data_ptr(), _native.DTYPE_CODE[v.dtype],
                v.stride(0), n, H, sm_scale, out.data_ptr(), H * D, work.data_ptr(), work.numel(), _native.stream()))
    return out
