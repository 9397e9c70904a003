"""wdl_w4a4_linear_noalloc: the W4A4 linear for callers that cannot allocate device memory (a native host with a
fixed device-memory budget, or a streaming loop that must never call cudaMalloc / cudaFree because they can
synchronize the device), whose scratch is a fixed array inside the library instead of a caller workspace.

Checked through the C ABI against the existing entry point (wdl_w4a4_linear with a workspace) on the same
inputs, for two calls in a row (the shared array keeps the first call's contents; the second must not depend on
them), and the size limit rejected with a clear error before anything runs. This file sorts last so that a run
stopping at its first failure has already run every other test; it also passes alone in a fresh process."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.float().cpu().numpy().astype(np.float64), b.float().cpu().numpy().astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_noalloc_linear_matches_the_workspace_entry_point_twice():
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.quantization import w4a4
    lib = _native.lib()
    g = torch.Generator().manual_seed(21)
    M, K, N = 1392, 3072, 3072
    W = torch.randn(N, K, generator=g) * 0.02
    layer = w4a4.PreparedW4A4(*(w4a4.quantize(W.cuda(), torch.randn(N, generator=g).cuda() * 0.1, rank=0,
                                              scale_dtype=torch.float16)[p] for p in w4a4.PARTS))
    st = _native.stream()
    for call in range(2):  # a different input each time: the second call must not see the first one's scratch
        x = (torch.randn(M, K, generator=g) * (1 + call)).to(torch.bfloat16).cuda()
        expected = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        work = torch.empty(lib.wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device="cuda")
        _native.check(lib.wdl_w4a4_linear(x.data_ptr(), K, M, K, None, _native.BF16, layer.codes.data_ptr(),
                                          layer.scales.data_ptr(), layer.code_format, layer.bias.data_ptr(), N,
                                          expected.data_ptr(), N, work.data_ptr(), work.numel(), st))
        got = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        _native.check(lib.wdl_w4a4_linear_noalloc(x.data_ptr(), K, M, K, None, _native.BF16, layer.codes.data_ptr(),
                                                  layer.scales.data_ptr(), layer.code_format, layer.bias.data_ptr(), N,
                                                  got.data_ptr(), N, st))
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert rel(got, expected) <= 2e-3
        assert torch.equal(got, expected)  # same kernels, same arithmetic: identical bits
    assert _native.device_error() == 0


def test_noalloc_linear_rejects_sizes_beyond_its_scratch():
    from wan_dit_lab_b200 import _native
    lib = _native.lib()
    K, N = 14336, 3072
    M = 2 * (16 << 20) // K  # about twice what the fixed scratch holds
    x = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(N, K, dtype=torch.uint8, device="cuda")
    ws = torch.ones(K // 64, N, device="cuda")
    y = torch.full((M, N), 7.0, dtype=torch.bfloat16, device="cuda")
    status = lib.wdl_w4a4_linear_noalloc(x.data_ptr(), K, M, K, None, _native.BF16, w.data_ptr(), ws.data_ptr(),
                                         _native.CODES_E4M3, None, N, y.data_ptr(), N, _native.stream())
    assert status == _native.ERR_ARGUMENT
    assert b"16 MiB" in lib.wdl_last_error()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # nothing ran
