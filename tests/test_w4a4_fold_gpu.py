"""The folded float16 code format (WDL_CODES_F16_FOLD): activation codes as float16 integers, weights folded with
their bf16 group scales and one power of two (wdl_w4a4_fold_weight), and the kind::f16 GEMM whose epilogue is
one fused multiply-add per element and group. Every folded weight must be exact, and the GEMM's outputs must
equal the E4M3 format's bit for bit (the same exact products, rounded once in the same order)."""

import math

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import w4a4 as ow

pytestmark = pytest.mark.gpu

E4M3, FOLD = 1, 3


def native():
    from wan_dit_lab_b200 import _native
    return _native


def random_codes(shape, seed, unsigned=False):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0 if unsigned else -8, 16 if unsigned else 8, shape, generator=g, dtype=torch.int8)


def scales(groups, rows, seed, lo, hi, dtype="bfloat16"):
    g = torch.Generator().manual_seed(seed)
    return ow.round_to((torch.rand(groups, rows, generator=g) * (hi - lo) + lo).numpy(), dtype)


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def fold(w_codes, sw_bf16):
    """Folded weights of integer codes [N, K] and bf16 scales [K/64, N] through the C ABI: (w16, 2^F tensor)."""
    _native = native()
    N, K = w_codes.shape
    packed = cu(ow.pack_nibbles(w_codes.numpy()))
    ws = torch.from_numpy(np.ascontiguousarray(sw_bf16)).to(torch.bfloat16).cuda()
    shift = math.ceil(math.log2(8 * float(np.abs(sw_bf16).max()))) - 15
    w16 = torch.empty(N, K, dtype=torch.float16, device="cuda")
    inexact = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(_native.lib().wdl_w4a4_fold_weight(packed.data_ptr(), ws.data_ptr(), _native.BF16, N, K, shift,
                                                     w16.data_ptr(), inexact.data_ptr(), _native.stream()))
    assert int(inexact.item()) == 0
    return w16, torch.tensor([2.0 ** shift], device="cuda"), shift


def test_fold_weight_exact():
    N, K = 384, 512
    w = random_codes((N, K), 1)
    sw = scales(K // 64, N, 2, 1e-4, 0.05)
    w16, _, shift = fold(w, sw)
    expected = (w.numpy().astype(np.float64) * np.repeat(sw.T.astype(np.float64), 64, axis=1) * 2.0 ** -shift)
    np.testing.assert_array_equal(w16.float().cpu().numpy().astype(np.float64), expected)
    assert np.abs(expected).max() <= 2 ** 15


def test_fold_weight_reports_inexact_f16_scales():
    """float16 scales carry 11 significant bits: code * scale needs up to 14, not a float16 number."""
    _native = native()
    N, K = 256, 128
    packed = cu(ow.pack_nibbles(random_codes((N, K), 3).numpy()))
    ws = (torch.rand(K // 64, N, generator=torch.Generator().manual_seed(4)) * 0.01 + 0.001).to(torch.float16).cuda()
    w16 = torch.empty(N, K, dtype=torch.float16, device="cuda")
    inexact = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(_native.lib().wdl_w4a4_fold_weight(packed.data_ptr(), ws.data_ptr(), _native.F16, N, K, -12,
                                                     w16.data_ptr(), inexact.data_ptr(), _native.stream()))
    assert int(inexact.item()) > 0


@pytest.mark.parametrize("M,K,dtype", [(300, 1024, torch.bfloat16), (37, 256, torch.float32)])
def test_quantizers_write_float16_codes(M, K, dtype):
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(M, K, generator=g) * 3).to(dtype).cuda()
    c_int, s_int = w4a4.quantize_rows(x, torch.bfloat16, code_format="int8")
    c16, s16 = w4a4.quantize_rows(x, torch.bfloat16, code_format="f16fold")
    assert c16.dtype == torch.float16
    assert torch.equal(c16.float(), c_int.float()) and torch.equal(s16, s_int)
    if dtype == torch.float32 and K >= 256:
        out = {}
        for fmt in (E4M3, FOLD):
            codes = torch.empty(M, K * 2, dtype=torch.uint8, device="cuda")
            sc = torch.empty(K // 64, M, device="cuda")
            _native.check(_native.lib().wdl_ln_quant(x.data_ptr(), _native.F32, K, M, K, 1e-6, None, None, 0, None,
                                                     None, None, _native.BF16, fmt, codes.data_ptr(), sc.data_ptr(),
                                                     _native.stream()))
            vals = (codes.view(-1)[: M * K * 2].view(torch.float16) if fmt == FOLD
                    else codes.view(-1)[: M * K].view(torch.float8_e4m3fn))
            out[fmt] = (vals.float().view(M, K).cpu(), sc.cpu())
        assert torch.equal(out[E4M3][0], out[FOLD][0]) and torch.equal(out[E4M3][1], out[FOLD][1])


@pytest.mark.parametrize("M,N,K,unsigned", [(300, 768, 1024, False), (1, 256, 128, False), (1392, 9216, 3072, False),
                                            (200, 3072, 14336, True), (129, 512, 192, False)])
def test_gemm_bit_identical_to_e4m3(M, N, K, unsigned):
    _native = native()
    lib = _native.lib()
    a, w = random_codes((M, K), 6, unsigned), random_codes((N, K), 7)
    sa, sw = scales(K // 64, M, 8, 0.01, 0.5), scales(K // 64, N, 9, 1e-4, 0.01)
    bias = cu((torch.randn(N, generator=torch.Generator().manual_seed(10)) * 0.1).numpy())
    sac, swc = cu(sa), cu(sw)
    ys = {}
    if K % 128 == 0:  # the E4M3 kernel's tile depth
        ae, we = cu(of.to_e4m3_bits(a.numpy().astype(np.float32))), cu(of.to_e4m3_bits(w.numpy().astype(np.float32)))
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        _native.check(lib.wdl_w4a4_gemm(ae.data_ptr(), sac.data_ptr(), we.data_ptr(), swc.data_ptr(), E4M3,
                                        bias.data_ptr(), M, N, K, y.data_ptr(), N, _native.stream()))
        ys[E4M3] = y.cpu()
    a16 = a.to(torch.float16).cuda()
    w16, f, _ = fold(w, sw)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _native.check(lib.wdl_w4a4_gemm(a16.data_ptr(), sac.data_ptr(), w16.data_ptr(), f.data_ptr(), FOLD,
                                    bias.data_ptr(), M, N, K, y.data_ptr(), N, _native.stream()))
    ys[FOLD] = y.cpu()
    if E4M3 in ys:
        assert torch.equal(ys[E4M3], ys[FOLD])
    expected = ow.gemm(a.numpy(), sa, w.numpy(), sw, bias.cpu().numpy())
    got = ys[FOLD].float().numpy()
    assert float(np.linalg.norm(got - expected) / np.linalg.norm(expected)) <= 2e-3
    assert _native.device_error() == 0


def test_residual_and_gelu_epilogues_bit_identical():
    _native = native()
    lib = _native.lib()
    M, N, K = 257, 512, 768
    a, w = random_codes((M, K), 11), random_codes((N, K), 12)
    sa, sw = scales(K // 64, M, 13, 0.01, 0.5), scales(K // 64, N, 14, 1e-4, 0.01)
    g = torch.Generator().manual_seed(15)
    bias, gate = (torch.randn(N, generator=g) * 0.1).cuda(), torch.randn(N, generator=g).cuda()
    res = torch.randn(M, N, generator=g).cuda()
    smooth = (torch.rand(N, generator=g) + 0.5).to(torch.bfloat16).cuda()
    sac, swc = cu(sa), cu(sw)
    ae, we = cu(of.to_e4m3_bits(a.numpy().astype(np.float32))), cu(of.to_e4m3_bits(w.numpy().astype(np.float32)))
    a16 = a.to(torch.float16).cuda()
    w16, f, _ = fold(w, sw)
    out = {}
    for fmt, (A, W, S) in ((E4M3, (ae, we, swc)), (FOLD, (a16, w16, f))):
        r = []
        for gp in (gate.data_ptr(), None):
            o = torch.empty(M, N, device="cuda")
            _native.check(lib.wdl_w4a4_gemm_residual(A.data_ptr(), sac.data_ptr(), W.data_ptr(), S.data_ptr(), fmt,
                                                     bias.data_ptr(), gp, res.data_ptr(), N, M, N, K, o.data_ptr(), N,
                                                     _native.stream()))
            r.append(o.cpu())
        codes = torch.empty(M, N * 2, dtype=torch.uint8, device="cuda")
        hs = torch.zeros(N // 64, M, device="cuda")
        _native.check(lib.wdl_w4a4_gemm_gelu_u4(A.data_ptr(), sac.data_ptr(), W.data_ptr(), S.data_ptr(), fmt,
                                                bias.data_ptr(), smooth.data_ptr(), 0.171875, _native.BF16, M, N, K,
                                                codes.data_ptr(), N, hs.data_ptr(), _native.stream()))
        vals = (codes.view(-1)[: M * N * 2].view(torch.float16) if fmt == FOLD
                else codes.view(-1)[: M * N].view(torch.float8_e4m3fn))
        r += [vals.float().view(M, N).cpu(), hs.cpu()]
        out[fmt] = r
    for x, y in zip(out[E4M3], out[FOLD]):
        assert torch.equal(x, y)
    assert _native.device_error() == 0


def test_prepared_layer_folds_bf16_and_falls_back_for_f16_scales():
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    K, N, M = 3072, 3072, 600
    g = torch.Generator().manual_seed(16)
    W = (torch.randn(N, K, generator=g) * 0.02).cuda()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    parts = w4a4.quantize(W, rank=0, scale_dtype=torch.bfloat16)
    e = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format="e4m3")
    f = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format="f16fold")
    assert f.code_format == _native.CODES_F16_FOLD
    assert torch.equal(e(x), f(x))
    parts16 = w4a4.quantize(W, rank=0, scale_dtype=torch.float16)
    f16 = w4a4.PreparedW4A4(*(parts16[p] for p in w4a4.PARTS), code_format="f16fold")
    assert f16.code_format == _native.CODES_E4M3
