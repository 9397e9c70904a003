"""The padded-scale code format (WDL_CODES_E4M3_TS): E4M3 codes, every group scale stored as (s, 0, 0, 0), and
the GEMM that forms the products of activation and weight scales on the tensor cores (a rank-1 tf32 MMA per
group) next to the FP8 group partials. Its results must equal the E4M3 format's bit for bit (the product of two
bf16/f16 scales is exact either way and the promotion does the same fused multiply-add in the same order), the
group partials must equal the exact integer sums, and the quantizers must write the same codes and scales."""

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import w4a4 as ow

pytestmark = pytest.mark.gpu

TS, E4M3 = 2, 1


def native():
    from wan_dit_lab_b200 import _native
    return _native


def padded(scales):
    """[G, rows] float32 -> [G, rows, 4] holding (s, 0, 0, 0)."""
    s = np.asarray(scales, np.float32)
    out = np.zeros(s.shape + (4,), np.float32)
    out[..., 0] = s
    return out


def random_codes(shape, seed, unsigned=False):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0 if unsigned else -8, 16 if unsigned else 8, shape, generator=g, dtype=torch.int8)


def e4m3(codes):
    return torch.from_numpy(np.ascontiguousarray(of.to_e4m3_bits(codes.numpy().astype(np.float32)))).cuda()


def scales(groups, rows, seed, lo, hi, dtype="bfloat16"):
    g = torch.Generator().manual_seed(seed)
    return ow.round_to((torch.rand(groups, rows, generator=g) * (hi - lo) + lo).numpy(), dtype)


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("M,K,dtype", [(300, 1024, torch.bfloat16), (37, 256, torch.float32), (1, 64, torch.bfloat16)])
@pytest.mark.parametrize("scale_dtype", [torch.bfloat16, torch.float16])
def test_quantize_rows_padded(M, K, dtype, scale_dtype):
    from wan_dit_lab_b200.quantization import w4a4
    g = torch.Generator().manual_seed(12)
    x = (torch.randn(M, K, generator=g) * 3).to(dtype).cuda()
    c1, s1 = w4a4.quantize_rows(x, scale_dtype, code_format="e4m3")
    c2, s2 = w4a4.quantize_rows(x, scale_dtype, code_format="e4m3ts")
    assert s2.shape == (K // 64, M, 4)
    assert torch.equal(c1, c2)
    np.testing.assert_array_equal(s2.cpu().numpy(), padded(s1.cpu().numpy()))


def test_ln_quant_padded():
    _native = native()
    M, K = 200, 3072
    g = torch.Generator().manual_seed(13)
    x = torch.randn(M, K, generator=g).cuda()
    shift, scale = (torch.randn(K, generator=g) * 0.1).cuda(), (torch.randn(K, generator=g) * 0.1).cuda()
    out = {}
    for fmt in (E4M3, TS):
        codes = torch.empty(M, K, dtype=torch.uint8, device="cuda")
        sc = torch.zeros(K // 64, M, 4, device="cuda")
        _native.check(_native.lib().wdl_ln_quant(x.data_ptr(), _native.F32, K, M, K, 1e-6, None, None, 0,
                                                 shift.data_ptr(), scale.data_ptr(), None, _native.BF16, fmt,
                                                 codes.data_ptr(), sc.data_ptr(), _native.stream()))
        out[fmt] = (codes.cpu(), sc.cpu().numpy())
    assert torch.equal(out[E4M3][0], out[TS][0])
    compact = out[E4M3][1].reshape(-1)[: K // 64 * M].reshape(K // 64, M)
    np.testing.assert_array_equal(out[TS][1], padded(compact))


def test_unpack_weight_padded():
    _native = native()
    N, K = 384, 512
    g = torch.Generator().manual_seed(14)
    packed = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8).cuda()
    ws = (torch.rand(K // 64, N, generator=g) * 0.01).to(torch.float16).cuda()
    codes = torch.empty(N, K, dtype=torch.uint8, device="cuda")
    sc = torch.empty(K // 64, N, 4, device="cuda")
    _native.check(_native.lib().wdl_w4a4_unpack_weight(packed.data_ptr(), ws.data_ptr(), _native.F16, N, K, TS,
                                                       codes.data_ptr(), sc.data_ptr(), _native.stream()))
    np.testing.assert_array_equal(codes.cpu().numpy(),
                                  of.to_e4m3_bits(ow.unpack_nibbles(packed.cpu().numpy()).astype(np.float32)))
    np.testing.assert_array_equal(sc.cpu().numpy(), padded(ws.float().cpu().numpy()))


@pytest.mark.parametrize("M,N,K,groups,unsigned", [(300, 384, 512, (0, 3, 7), False), (1392, 9216, 3072, (0, 47), False),
                                                   (129, 256, 1024, (0, 15), True)])
def test_group_partials_bit_exact(M, N, K, groups, unsigned):
    _native = native()
    a, w = random_codes((M, K), 1, unsigned), random_codes((N, K), 2)
    sa, sw = cu(padded(np.ones((K // 64, M)))), cu(padded(np.ones((K // 64, N))))
    ac, wc = e4m3(a), e4m3(w)
    out = torch.empty(M, N, dtype=torch.int32, device="cuda")
    for group in groups:
        _native.check(_native.lib().wdl_w4a4_gemm_group_partials(
            ac.data_ptr(), sa.data_ptr(), wc.data_ptr(), sw.data_ptr(), TS, M, N, K, group, out.data_ptr(), N,
            _native.stream()))
        np.testing.assert_array_equal(out.cpu().numpy(), ow.group_partials(a.numpy(), w.numpy(), [group])[0])
    assert _native.device_error() == 0


@pytest.mark.parametrize("M,N,K,sdt", [(300, 768, 1024, "bfloat16"), (1, 256, 128, "bfloat16"),
                                       (1392, 9216, 3072, "bfloat16"), (200, 3072, 14336, "float16"),
                                       (129, 1024, 256, "float16")])
def test_gemm_bit_identical_to_cuda_core_promotion(M, N, K, sdt):
    _native = native()
    lib = _native.lib()
    a, w = random_codes((M, K), 3), random_codes((N, K), 4)
    sa = scales(K // 64, M, 5, 0.01, 0.5)
    sw = scales(K // 64, N, 6, 1e-4, 0.01, sdt)
    bias = cu((torch.randn(N, generator=torch.Generator().manual_seed(7)) * 0.1).numpy())
    ac, wc = e4m3(a), e4m3(w)
    ys = {}
    for fmt, (s_a, s_w) in ((E4M3, (cu(sa), cu(sw))), (TS, (cu(padded(sa)), cu(padded(sw))))):
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        _native.check(lib.wdl_w4a4_gemm(ac.data_ptr(), s_a.data_ptr(), wc.data_ptr(), s_w.data_ptr(), fmt,
                                        bias.data_ptr(), M, N, K, y.data_ptr(), N, _native.stream()))
        ys[fmt] = y.cpu()
    assert torch.equal(ys[E4M3], ys[TS])
    expected = ow.gemm(a.numpy(), sa, w.numpy(), sw, bias.cpu().numpy())
    got = ys[TS].float().numpy()
    assert float(np.linalg.norm(got - expected) / np.linalg.norm(expected)) <= 2e-3
    assert _native.device_error() == 0


def test_gemm_n_multiple_of_128_only():
    """N = 384 runs only on the padded-scale kernel (128-column tiles); checked against the oracle."""
    _native = native()
    M, N, K = 257, 384, 640
    a, w = random_codes((M, K), 8), random_codes((N, K), 9)
    sa, sw = scales(K // 64, M, 10, 0.01, 0.5), scales(K // 64, N, 11, 1e-4, 0.01)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    s_a, s_w = cu(padded(sa)), cu(padded(sw))
    ac, wc = e4m3(a), e4m3(w)  # held: a temporary's memory could be reused before the kernel reads it
    _native.check(_native.lib().wdl_w4a4_gemm(ac.data_ptr(), s_a.data_ptr(), wc.data_ptr(), s_w.data_ptr(),
                                               TS, None, M, N, K, y.data_ptr(), N, _native.stream()))
    expected = ow.round_to(ow.gemm(a.numpy(), sa, w.numpy(), sw), "bfloat16")
    got = y.float().cpu().numpy()
    assert float(np.linalg.norm(got - expected) / np.linalg.norm(expected)) <= 1e-3


def test_residual_and_gelu_epilogues_bit_identical():
    _native = native()
    lib = _native.lib()
    M, N, K = 257, 512, 768
    a, w = random_codes((M, K), 12), random_codes((N, K), 13)
    sa, sw = scales(K // 64, M, 14, 0.01, 0.5), scales(K // 64, N, 15, 1e-4, 0.01)
    g = torch.Generator().manual_seed(16)
    bias, gate = (torch.randn(N, generator=g) * 0.1).cuda(), torch.randn(N, generator=g).cuda()
    res = torch.randn(M, N, generator=g).cuda()
    smooth = (torch.rand(N, generator=g) + 0.5).to(torch.bfloat16).cuda()
    ac, wc = e4m3(a), e4m3(w)
    out = {}
    for fmt, (s_a, s_w) in ((E4M3, (cu(sa), cu(sw))), (TS, (cu(padded(sa)), cu(padded(sw))))):
        r = []
        for gp in (gate.data_ptr(), None):
            o = torch.empty(M, N, device="cuda")
            _native.check(lib.wdl_w4a4_gemm_residual(ac.data_ptr(), s_a.data_ptr(), wc.data_ptr(), s_w.data_ptr(), fmt,
                                                     bias.data_ptr(), gp, res.data_ptr(), N, M, N, K, o.data_ptr(), N,
                                                     _native.stream()))
            r.append(o.cpu())
        codes = torch.empty(M, N, dtype=torch.uint8, device="cuda")
        hs = torch.zeros(N // 64, M, 4, device="cuda")
        _native.check(lib.wdl_w4a4_gemm_gelu_u4(ac.data_ptr(), s_a.data_ptr(), wc.data_ptr(), s_w.data_ptr(), fmt,
                                                bias.data_ptr(), smooth.data_ptr(), 0.171875, _native.BF16, M, N, K,
                                                codes.data_ptr(), N, hs.data_ptr(), _native.stream()))
        hsn = hs.cpu().numpy()
        r += [codes.cpu(), hsn[..., 0] if fmt == TS else hsn.reshape(-1)[: N // 64 * M].reshape(N // 64, M)]
        if fmt == TS:
            assert not hsn[..., 1:].any()
        out[fmt] = r
    for x, y in zip(out[E4M3][:3], out[TS][:3]):
        assert torch.equal(x, y)
    np.testing.assert_array_equal(out[E4M3][3], out[TS][3])
    assert _native.device_error() == 0


@pytest.mark.parametrize("M", [1392, 37])
def test_packed_linear_config1(M):
    """BASELINE config 1 through PreparedW4A4: the padded-scale format equals the E4M3 format bit for bit."""
    from wan_dit_lab_b200.quantization import w4a4
    K, N = 3072, 9216
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=g)
    x[:, torch.randperm(K, generator=g)[:30]] *= 20
    W = torch.randn(N, K, generator=g) * 0.02
    parts = w4a4.quantize(W.cuda(), rank=0, scale_dtype=torch.float16)
    ys = [w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=f)(x.to(torch.bfloat16).cuda()).cpu()
          for f in ("e4m3", "e4m3ts")]
    assert torch.equal(ys[0], ys[1])


def test_noalloc_linear_padded_scales():
    _native = native()
    from wan_dit_lab_b200.quantization import w4a4
    lib = _native.lib()
    M, K, N = 600, 3072, 3072
    g = torch.Generator().manual_seed(17)
    layer = w4a4.PreparedW4A4(*(w4a4.quantize((torch.randn(N, K, generator=g) * 0.02).cuda(), rank=0)[p]
                                for p in w4a4.PARTS), code_format="e4m3ts")
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    y1, y2 = (torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    work = torch.empty(lib.wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device="cuda")
    _native.check(lib.wdl_w4a4_linear(x.data_ptr(), K, M, K, None, _native.BF16, layer.codes.data_ptr(),
                                      layer.scales.data_ptr(), TS, None, N, y1.data_ptr(), N, work.data_ptr(),
                                      work.numel(), _native.stream()))
    _native.check(lib.wdl_w4a4_linear_noalloc(x.data_ptr(), K, M, K, None, _native.BF16, layer.codes.data_ptr(),
                                              layer.scales.data_ptr(), TS, None, N, y2.data_ptr(), N, _native.stream()))
    assert torch.equal(y1, y2)
