"""RoPE, the FP8 KV-cache store and the fused QKV preparation on the B200 kernels against the CPU oracle, with
the contract tests of the reference (tests/test_cache_fp8.py, tests/test_rope_triton.py): bitwise values and
scales, untouched cache outside the written rows, unmodified inputs, strided inputs and mixed dtypes, another
stream, boundary values, and invalid contracts rejected before any write."""

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import rope as orope

pytestmark = pytest.mark.gpu


def kv():
    from wan_dit_lab_b200.kernels import cache_fp8
    return cache_fp8


def buffers(batch, tokens, heads, dim):
    shape = (batch, tokens, heads, dim)
    return (torch.full(shape, 2., device="cuda").to(torch.float8_e4m3fn),
            torch.full((batch, tokens, heads, 1), 7., device="cuda"),
            torch.full(shape, -2., device="cuda").to(torch.float8_e4m3fn),
            torch.full((batch, tokens, heads, 1), 9., device="cuda"))


def expect_store(bufs, at, k, v):
    """The oracle's cache after storing k, v at `at` into copies of bufs."""
    ck, cks, cv, cvs = (b.cpu() for b in bufs)
    ck, cv = ck.view(torch.uint8).numpy().copy(), cv.view(torch.uint8).numpy().copy()
    cks, cvs = cks.numpy().copy(), cvs.numpy().copy()
    n = k.shape[1]
    ck[:, at:at + n], cks[:, at:at + n] = of.quantize_rows(k.float().cpu().numpy())
    cv[:, at:at + n], cvs[:, at:at + n] = of.quantize_rows(v.float().cpu().numpy())
    return ck, cks, cv, cvs


def assert_cache(bufs, expected):
    got = (bufs[0].view(torch.uint8).cpu().numpy(), bufs[1].cpu().numpy(), bufs[2].view(torch.uint8).cpu().numpy(),
           bufs[3].cpu().numpy())
    for g, e in zip(got, expected):
        np.testing.assert_array_equal(g, e)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("batch,heads,dim", [(1, 2, 64), (2, 3, 128), (1, 1, 160)])
def test_store_bitwise_values_scales_and_untouched_cache(dtype, batch, heads, dim):
    torch.manual_seed(23)
    k = torch.randn(batch, 7, heads, dim, device="cuda", dtype=dtype)
    v = torch.randn_like(k)
    actual = buffers(batch, 17, heads, dim)
    expected = expect_store(actual, 5, k, v)
    before_k, before_v = k.clone(), v.clone()
    kv().store_kv_fp8(k, v, *actual, 5)
    assert_cache(actual, expected)
    assert torch.equal(k, before_k) and torch.equal(v, before_v)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_store_zero_tiny_large_and_fp8_rounding_boundaries(dtype):
    values = torch.tensor([0., -0., 1e-15, -1e-15, .5, -.5, 1., -1., 3., -3., 448., -448.], device="cuda").to(dtype)
    k = values.repeat(8).reshape(1, 1, 1, 96)
    v = torch.zeros_like(k)
    actual = buffers(1, 3, 1, 96)
    expected = expect_store(actual, 1, k, v)
    kv().store_kv_fp8(k, v, *actual, 1)
    assert_cache(actual, expected)


def test_store_fp32_values_around_fp8_midpoints():
    # 84.021 -> 84 in FP16 -> 80 in FP8, but direct FP32 -> FP8 is 88 (reference test_cache_fp8.py:150-158)
    k = torch.tensor([448., 84.021, -84.021, 1.06251, -1.06251, 1.06249, -1.06249, 0.], device="cuda").reshape(1, 1, 1, 8)
    actual = buffers(1, 3, 1, 8)
    expected = expect_store(actual, 1, k, k)
    kv().store_kv_fp8(k, k, *actual, 1)
    assert_cache(actual, expected)


def test_store_strided_inputs_mixed_dtypes_and_nondefault_stream():
    k = torch.randn(2, 5, 3, 256, device="cuda", dtype=torch.float32)[..., ::2]
    v = torch.randn(2, 10, 3, 128, device="cuda", dtype=torch.bfloat16)[:, ::2]
    actual = buffers(2, 11, 3, 128)
    expected = expect_store(actual, 6, k, v)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        kv().store_kv_fp8(k, v, *actual, 6)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    assert_cache(actual, expected)


def test_store_captured_in_a_cuda_graph():
    k = torch.randn(1, 7, 2, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    actual = buffers(1, 12, 2, 128)
    kv().store_kv_fp8(k, v, *actual, 4)  # first call outside capture (library load)
    graph = torch.cuda.CUDAGraph()
    fresh = buffers(1, 12, 2, 128)
    for t, f in zip(actual, fresh):
        t.copy_(f)
    expected = expect_store(actual, 4, k, v)
    with torch.cuda.graph(graph):
        kv().store_kv_fp8(k, v, *actual, 4)
    graph.replay()
    torch.cuda.synchronize()
    assert_cache(actual, expected)


@pytest.mark.parametrize("problem", ["negative", "overflow", "shape", "cache_dtype", "scale_dtype", "grad"])
def test_store_invalid_contract_rejected_before_write(problem):
    k = torch.randn(1, 5, 2, 128, device="cuda")
    v, actual, offset = k.clone(), list(buffers(1, 8, 2, 128)), 1
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
    else:
        k.requires_grad_()
    before = [t.clone() for t in actual]
    with pytest.raises((ValueError, TypeError)):
        kv().store_kv_fp8(k, v, *actual, offset)
    for t, b in zip(actual, before):
        assert torch.equal(t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t,
                           b.view(torch.uint8) if b.dtype == torch.float8_e4m3fn else b)


# ---- RoPE


def frequencies(dim=128, positions=64, dtype=np.float64):
    pairs = dim // 2
    spatial = pairs // 3
    return np.concatenate([orope.rope(positions, 2 * n) for n in (pairs - 2 * spatial, spatial, spatial)],
                          axis=-1).astype(dtype)


def oracle_rope(x, grids, freq, start, out_dtype):
    x = x.detach().cpu()
    xn = x.double().numpy() if x.dtype == torch.float64 else x.float().numpy()
    name = str(out_dtype).split(".")[1]
    work = np.float64 if (x.dtype == torch.float64 or freq.dtype == np.float64) else np.float32
    outs = []
    for b, g in enumerate(grids):
        o = orope.rope_apply(xn[b:b + 1].astype(work), tuple(g), freq.astype(work), start, out_dtype=name)
        outs.append(o)
    return np.concatenate(outs, axis=0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
@pytest.mark.parametrize("table", [np.float32, np.float64])
@pytest.mark.parametrize("batch", [1, 2, 4])
def test_rope_bitwise_same_shape_batches(dtype, table, batch):
    from wan_dit_lab_b200.kernels.rope import rope_apply
    torch.manual_seed(12)
    grids = ((2, 3, 5),) * batch
    x = torch.randn(batch, 30, 3, 128, device="cuda", dtype=dtype)
    freq = frequencies(dtype=table)
    actual = rope_apply(x, grids, torch.from_numpy(freq).cuda(), 7)
    expected = oracle_rope(x, grids, freq, 7, dtype)
    np.testing.assert_array_equal(actual.cpu().double().numpy() if dtype == torch.float64 else actual.float().cpu().numpy(),
                                  expected)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_rope_strided_input_heterogeneous_grids_padding_and_no_mutation(dtype):
    from wan_dit_lab_b200.kernels.rope import rope_apply
    grids = ((2, 3, 5), (1, 2, 4))
    x = torch.randn(2, 33, 2, 256, device="cuda", dtype=dtype)[..., ::2]
    before = x.clone()
    freq = frequencies(dtype=np.float32)
    actual = rope_apply(x, torch.tensor(grids), torch.from_numpy(freq).cuda(), 3)
    np.testing.assert_array_equal(actual.float().cpu().numpy(), oracle_rope(x, grids, freq, 3, dtype))
    assert torch.equal(x, before)
    for b, (f, h, w) in enumerate(grids):
        assert torch.equal(actual[b, f * h * w:], x[b, f * h * w:])
    assert actual.dtype == x.dtype and actual.shape == x.shape and actual.data_ptr() != x.data_ptr()


@pytest.mark.parametrize("problem", ["odd_dim", "grid_count", "grid_length", "negative_start", "frequency_bounds",
                                     "frequency_grad"])
def test_rope_invalid_contract_is_rejected(problem):
    from wan_dit_lab_b200.kernels.rope import rope_apply
    x = torch.randn(1, 6, 1, 12, device="cuda")
    grids, start, freq = ((1, 2, 3),), 0, torch.from_numpy(frequencies(12)).cuda()
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
    else:
        freq.requires_grad_()
    with pytest.raises((ValueError, TypeError)):
        rope_apply(x, grids, freq, start)


# ---- fused QKV preparation


@pytest.mark.parametrize("n,dim,grid,start,at", [(2 * 4 * 8, 1024, (4, 8), 3, 64), (1392, 3072, (16, 29), 9, 4176)])
def test_qkv_prep_matches_oracle_chain(n, dim, grid, start, at):
    """RMSNorm(q), RMSNorm(k) -> RoPE -> FP8 store, against the oracle's chain on the same inputs."""
    from wan_dit_lab_b200 import _native
    g = torch.Generator().manual_seed(5)
    heads = dim // 128
    qkv = torch.randn(n, 3 * dim, generator=g).to(torch.bfloat16)
    wq = torch.randn(dim, generator=g) * 0.1 + 1.0
    wk = torch.randn(dim, generator=g) * 0.1 + 1.0
    positions = 1024
    freq = frequencies(128, positions, np.float32)
    cap = at + n + 16
    ck = torch.zeros(cap, heads, 128, dtype=torch.uint8, device="cuda")
    cv = torch.zeros_like(ck)
    cks = torch.zeros(cap, heads, device="cuda")
    cvs = torch.zeros_like(cks)
    q_out = torch.empty(n, dim, device="cuda")
    k_out = torch.empty(n, dim, device="cuda")
    d_qkv, d_wq, d_wk, d_f = qkv.cuda(), wq.cuda(), wk.cuda(), torch.from_numpy(freq).cuda()
    _native.check(_native.lib().wdl_qkv_prep(
        d_qkv.data_ptr(), 3 * dim, n, dim, d_wq.data_ptr(), d_wk.data_ptr(), 1e-6, d_f.data_ptr(), positions, grid[0],
        grid[1], start, q_out.data_ptr(), k_out.data_ptr(), ck.data_ptr(), cks.data_ptr(), cv.data_ptr(),
        cvs.data_ptr(), cap, at, _native.stream()))
    x = qkv.float().numpy()
    frames = n // (grid[0] * grid[1])
    for part, w, out in ((0, wq, q_out), (1, wk, k_out)):
        normed = orope.rms_norm(x[:, part * dim:(part + 1) * dim], w.numpy(), round_to="bfloat16")
        rot = orope.rope_apply(normed.reshape(1, n, heads, 128), (frames, *grid), freq, start)[0].reshape(n, dim)
        got = out.cpu().numpy()
        exact = (got == rot).mean()
        assert exact >= 0.999, exact  # RMSNorm's float32 sum in another order may move a bf16 rounding
        # one bf16 step of a normalized input (|x| ~ 1) moves a rotated value by up to ~2^-7 absolutely, and more
        # than that relatively where the rotation cancels
        np.testing.assert_allclose(got, rot, rtol=2 ** -7, atol=2 ** -6)
    # the stored rows are quantize_rows of the rotated keys the kernel produced, and of the raw values, bit for bit
    kq, ksc = of.quantize_rows(k_out.cpu().numpy().reshape(n, heads, 128))
    vq, vsc = of.quantize_rows(x[:, 2 * dim:].reshape(n, heads, 128))
    np.testing.assert_array_equal(ck[at:at + n].cpu().numpy(), kq)
    np.testing.assert_array_equal(cks[at:at + n].cpu().numpy(), ksc[..., 0])
    np.testing.assert_array_equal(cv[at:at + n].cpu().numpy(), vq)
    np.testing.assert_array_equal(cvs[at:at + n].cpu().numpy(), vsc[..., 0])
    assert int(ck[:at].count_nonzero()) == 0 and int(ck[at + n:].count_nonzero()) == 0
