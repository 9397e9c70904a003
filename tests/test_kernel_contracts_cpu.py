"""The Python operators' contracts without a GPU: invalid calls of store_kv_fp8, rope_apply and sage_kv.attend are
refused with the reference's exception types before anything is launched or written, as its own tests require
(tests/test_cache_fp8.py:113-129, tests/test_rope_triton.py:226-242). The tensors are fake CUDA tensors
(FakeTensorMode: shapes, dtypes and devices without memory), which is all the validation reads."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode


@pytest.fixture
def fake():
    with FakeTensorMode() as mode:
        yield mode


def cache_buffers(b, tokens, h, d):
    k = torch.zeros(b, tokens, h, d, device="cuda").to(torch.float8_e4m3fn)
    ks = torch.zeros(b, tokens, h, 1, device="cuda")
    return [k, ks, torch.zeros_like(k), torch.zeros_like(ks)]


STORE = dict(negative="cache bounds", overflow="cache bounds", shape="matching", cache_dtype="FP8 E4M3FN",
             scale_dtype="FP32", grad="inference-only", host_tensor="same CUDA device", cache_shape="Cache dimensions",
             strided_cache="contiguous")


@pytest.mark.parametrize("problem", list(STORE))
def test_store_kv_fp8_rejects_invalid_contracts(fake, problem):
    from wan_dit_lab_b200.kernels.cache_fp8 import store_kv_fp8
    k = torch.randn(1, 5, 2, 128, device="cuda")
    v, actual, offset = k.clone(), cache_buffers(1, 8, 2, 128), 1
    if problem == "negative":
        offset = -1
    elif problem == "overflow":
        offset = 4
    elif problem == "shape":
        v = v[:, :3]
    elif problem == "cache_dtype":
        actual[0] = actual[0].float()
    elif problem == "scale_dtype":
        actual[1] = actual[1].half()
    elif problem == "grad":
        k.requires_grad_()
    elif problem == "host_tensor":
        v = torch.randn(1, 5, 2, 128)
    elif problem == "cache_shape":
        actual[2] = torch.zeros(1, 8, 3, 128, device="cuda").to(torch.float8_e4m3fn)
    else:
        actual[0] = torch.zeros(1, 8, 2, 256, device="cuda").to(torch.float8_e4m3fn)[..., ::2]
    with pytest.raises((ValueError, TypeError), match=STORE[problem]):
        store_kv_fp8(k, v, *actual, offset)


ROPE = dict(odd_dim="even dim", grid_count="One grid", grid_length="exceeds sequence", negative_start="nonnegative",
            frequency_bounds="frequency bounds", frequency_grad="Trainable", frequency_dtype="FP32/FP64",
            grid_on_device="host metadata", output_dtype="output dtype")


@pytest.mark.parametrize("problem", list(ROPE))
def test_rope_apply_rejects_invalid_contracts(fake, problem):
    from wan_dit_lab_b200.kernels.rope import rope_apply
    x = torch.randn(1, 6, 1, 12, device="cuda")
    grids, start, freq, kw = ((1, 2, 3),), 0, torch.zeros(2, 64, 6, dtype=torch.float64, device="cuda"), {}
    if problem == "odd_dim":
        x = x[..., :11]
    elif problem == "grid_count":
        grids = grids * 2
    elif problem == "grid_length":
        grids = ((2, 2, 3),)
    elif problem == "negative_start":
        start = -1
    elif problem == "frequency_bounds":
        start = 64
    elif problem == "frequency_grad":
        freq.requires_grad_()
    elif problem == "frequency_dtype":
        freq = freq.to(torch.float16)
    elif problem == "grid_on_device":
        grids = torch.tensor([[1, 2, 3]], device="cuda")
    else:
        kw = dict(output_dtype=torch.int32)
    with pytest.raises((ValueError, TypeError), match=ROPE[problem]):
        rope_apply(x, grids, freq, start, **kw)


SAGE = dict(at_bounds="at exceeds", head_map_dtype="heads must be", token_map_length="tokens must be",
            cache_float="FP8 E4M3FN", batch="batch 1", head_dim="head_dim 128", chunk_dtype="float32 or bfloat16",
            scale_dtype="FP32")


@pytest.mark.parametrize("problem", list(SAGE))
def test_sage_attend_rejects_invalid_contracts(fake, problem):
    from wan_dit_lab_b200.kernels import sage_kv
    H, at, n = 2, 20, 10
    ck, cks, cv, cvs = cache_buffers(1, at + n, H, 128)
    Q = torch.randn(1, n, H, 128, device="cuda")
    K, V = torch.randn(1, n, H, 128, device="cuda"), torch.randn(1, n, H, 128, device="cuda").to(torch.bfloat16)
    kw = {}
    if problem == "at_bounds":
        at = 10 ** 6
    elif problem == "head_map_dtype":
        kw = dict(heads=torch.zeros(H, device="cuda"))
    elif problem == "token_map_length":
        kw = dict(tokens=torch.zeros(at - 1, dtype=torch.int32, device="cuda"))
    elif problem == "cache_float":
        ck = ck.float()
    elif problem == "batch":
        Q, K, V = (torch.cat([t, t]) for t in (Q, K, V))
    elif problem == "head_dim":
        Q, K, V = Q[..., :64], K[..., :64], V[..., :64]
    elif problem == "chunk_dtype":
        K = K.half()
        V = V.half()
    else:
        cks = cks.half()
    with pytest.raises((ValueError, TypeError), match=SAGE[problem]):
        sage_kv.attend(Q, ck, cks, cv, cvs, at, K, V, **kw)
