"""The prescaled float16 code format (WDL_CODES_F16_PRE): activations float16(code * stored scale * 2^-E_m), one
power of two per row, weights folded as in WDL_CODES_F16_FOLD; the GEMM accumulates all of K on the tensor cores.
The quantizers' values are exact (equal bit for bit to the folded format's codes times its scales, rescaled);
the GEMM equals the per-group promotion of the folded format within float32 rounding (bf16 outputs >= 99.9 %
bit-equal, relative L2 <= 2e-4: one bf16 step where the two float32 sums straddle a rounding boundary; the
float32 partial products within 1e-6), in every epilogue; the W4A4 linear stays within 2e-3 of the oracle."""

import numpy as np
import pytest
import torch

from oracle import w4a4 as ow

pytestmark = pytest.mark.gpu


def native():
    from wan_dit_lab_b200 import _native
    return _native


def seeded(shape, seed, scale=1.0, outliers=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    if outliers:
        cols = torch.randperm(shape[-1], generator=g)[: max(1, int(outliers * shape[-1]))]
        x[..., cols] *= 20
    return x


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def expected_prescaled(codes, scales, rows_scale):
    """float16(code * stored scale / 2^E_m) from the folded format's codes [M, K] and scales [K/64, M]."""
    per_col = scales.t().repeat_interleave(64, dim=1)  # [M, K]
    return (codes.float() * per_col / rows_scale[:, None]).half()


@pytest.mark.parametrize("M,K,smooth,dtype", [(300, 1024, False, torch.bfloat16), (129, 3072, True, torch.bfloat16),
                                              (37, 256, False, torch.float32)])
def test_quantize_rows_prescaled_values_exact(M, K, smooth, dtype):
    from wan_dit_lab_b200.quantization import w4a4
    x = seeded((M, K), 1, outliers=0.01).to(dtype).cuda()
    s = (seeded((K,), 2).abs() + 0.5).to(torch.bfloat16).cuda() if smooth else None
    c3, s3 = w4a4.quantize_rows(x, torch.bfloat16, smooth=s, code_format="f16fold")
    pre, rs = w4a4.quantize_rows(x, torch.bfloat16, smooth=s, code_format="f16pre")
    assert rs.shape == (M,)
    mant, _ = torch.frexp(rs)
    assert bool((mant == 0.5).all())  # powers of two
    top = s3.max(dim=0).values * 8 / rs  # 8 x the row's largest scale, rescaled: in [2^14, 2^15)
    assert bool(((top >= 2 ** 14) & (top < 2 ** 15)).all())
    want = expected_prescaled(c3, s3, rs)
    assert torch.equal(pre.view(torch.int16), want.view(torch.int16))


def test_ln_quant_prescaled_values_exact():
    _native = native()
    lib, st = _native.lib(), _native.stream()
    M, K = 200, 3072
    g = torch.Generator().manual_seed(3)
    X = torch.randn(M, K, generator=g).cuda()
    shift, scale = (torch.randn(K, generator=g) * 0.1).cuda(), (torch.randn(K, generator=g) * 0.1).cuda()
    smooth = (torch.rand(K, generator=g) + 0.5).to(torch.bfloat16).cuda()
    out = {}
    for fmt, shape in ((3, (K // 64, M)), (4, (M,))):
        codes = torch.empty(M, K, dtype=torch.float16, device="cuda")
        sc = torch.empty(shape, device="cuda")
        kept = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")  # the layer's bf16 input, before smoothing
        _native.check(lib.wdl_ln_quant_keep(X.data_ptr(), _native.F32, K, M, K, 1e-6, None, None, 0,
                                            shift.data_ptr(), scale.data_ptr(), smooth.data_ptr(), _native.BF16, fmt,
                                            codes.data_ptr(), sc.data_ptr(), kept.data_ptr(), K, st))
        out[fmt] = (codes, sc, kept)
    # the prescaled values are exactly the folded format's codes and scales of the layer input the kernel kept
    from wan_dit_lab_b200.quantization import w4a4
    c3, s3 = w4a4.quantize_rows(out[4][2], torch.bfloat16, smooth=smooth, code_format="f16fold")
    want = expected_prescaled(c3, s3, out[4][1])
    assert torch.equal(out[4][0].view(torch.int16), want.view(torch.int16))
    # both kernels' kept inputs: the LayerNorm statistics are float sums in different orders (two warps against
    # four per row), so a few bf16 values round the other way
    same = (out[4][2].view(torch.int16) == out[3][2].view(torch.int16)).float().mean().item()
    assert same >= 0.9999
    assert float((out[4][2].float() - out[3][2].float()).abs().max()) <= 2 ** -6 * float(out[3][2].float().abs().max())
    mean = X.mean(1, keepdim=True)
    ln = (X - mean) * torch.rsqrt(((X - mean) ** 2).mean(1, keepdim=True) + 1e-6)
    ref = (ln * (1 + scale) + shift).to(torch.bfloat16).float()
    assert float((out[4][2].float() - ref).abs().max()) <= 0.02 * float(ref.abs().max())


def prepared(N, K, seed):
    from wan_dit_lab_b200.quantization import w4a4
    W = seeded((N, K), seed, scale=0.02)
    b = seeded((N,), seed + 1, scale=0.1)
    parts = w4a4.quantize(W.cuda(), b.cuda(), rank=0)
    return (W, b, parts, w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format="f16fold"),
            w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format="f16pre"))


@pytest.mark.parametrize("M,N,K", [(300, 768, 1024), (1392, 3072, 3072), (64, 384, 512)])
def test_gemm_prescaled_matches_folded_in_every_epilogue(M, N, K):
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    lib, st = _native.lib(), _native.stream()
    x = seeded((M, K), 4, outliers=0.01).to(torch.bfloat16).cuda()
    _, _, _, fold, pre = prepared(N, K, 5)
    assert fold.code_format == 3 and pre.code_format == 4
    c3, s3 = w4a4.quantize_rows(x, torch.bfloat16, code_format="f16fold")
    c4, s4 = w4a4.quantize_rows(x, torch.bfloat16, code_format="f16pre")
    ops = {3: (c3, s3, fold), 4: (c4, s4, pre)}
    res = seeded((M, N), 6).cuda()
    gate = seeded((N,), 7).cuda()
    outs = {}
    for f, (c, s, L) in ops.items():
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        _native.check(lib.wdl_w4a4_gemm(c.data_ptr(), s.data_ptr(), L.codes.data_ptr(), L.scales.data_ptr(), f,
                                        L.bias.data_ptr(), M, N, K, y.data_ptr(), N, st))
        r = res.clone()
        _native.check(lib.wdl_w4a4_gemm_residual(c.data_ptr(), s.data_ptr(), L.codes.data_ptr(), L.scales.data_ptr(),
                                                 f, L.bias.data_ptr(), gate.data_ptr(), r.data_ptr(), N, M, N, K,
                                                 r.data_ptr(), N, st))
        p = torch.empty(M, N, device="cuda")
        _native.check(lib.wdl_w4a4_gemm_f32(c.data_ptr(), s.data_ptr(), L.codes.data_ptr(), L.scales.data_ptr(), f,
                                            None, None, 0, M, N, K, p.data_ptr(), N, st))
        hc = torch.empty(M, N, dtype=torch.float16, device="cuda")
        hs = torch.empty(N // 64, M, device="cuda")
        _native.check(lib.wdl_w4a4_gemm_gelu_u4(c.data_ptr(), s.data_ptr(), L.codes.data_ptr(), L.scales.data_ptr(),
                                                f, L.bias.data_ptr(), None, 0.171875, _native.BF16, M, N, K,
                                                hc.data_ptr(), N, hs.data_ptr(), st))
        outs[f] = (y, r, p, hc, hs)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    (y3, r3, p3, hc3, hs3), (y4, r4, p4, hc4, hs4) = outs[3], outs[4]
    assert rel(p4.cpu(), p3.cpu()) <= 1e-6
    # bf16 outputs: where the two float32 sums straddle a bf16 rounding boundary, one bf16 step apart
    assert rel(y4.float().cpu(), y3.float().cpu()) <= 2e-4 and (y4 == y3).float().mean().item() >= 0.999
    assert rel(r4.cpu(), r3.cpu()) <= 2e-4 and (r4 == r3).float().mean().item() >= 0.999
    assert (hc4 == hc3).float().mean().item() >= 0.999 and rel(hs4.cpu(), hs3.cpu()) <= 2e-4


def test_linear_prescaled_against_oracle():
    """BASELINE config 1's shapes with bf16 scales (the prescaled format's own): within 2e-3 of the oracle."""
    M, K, N = 1392, 3072, 9216
    x = seeded((M, K), 0, outliers=0.01).to(torch.bfloat16)
    W, _, parts, _, pre = prepared(N, K, 1)
    assert pre.code_format == 4
    y = pre(x.cuda()).float().cpu().numpy()
    o_codes = ow.unpack_nibbles(parts["qweight"].cpu().numpy())
    expected, _, _ = ow.linear(x.float().numpy(), o_codes, parts["wscales"].float().cpu().numpy(),
                               parts["bias"].float().cpu().numpy())
    assert rel(y, expected) <= 2e-3
    assert native().device_error() == 0


def test_block_prescaled_matches_folded_block():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from test_block_gpu import random_state
    from oracle import fp8 as of
    from oracle import rope as orope
    from wan_dit_lab_b200.models.block import Buffers, WanBlockB200
    dim, heads, ffn, frames, h, w, at, text = 1024, 8, 4096, 2, 4, 8, 128, 32
    n = frames * h * w
    state = random_state(dim, ffn, 9)
    g = torch.Generator().manual_seed(10)
    X = torch.randn(n, dim, generator=g)
    time_in = torch.randn(6, dim, generator=g) * 0.1
    ctx = torch.randn(text, dim, generator=g).to(torch.bfloat16)
    cap = at + n + 16
    ck8, cks = of.quantize_rows(torch.randn(1, cap, heads, 128, generator=g).numpy())
    cv8, cvs = of.quantize_rows(torch.randn(1, cap, heads, 128, generator=g).numpy())
    freq = torch.from_numpy(orope.table(1024).astype(np.float32)).cuda()
    outs = {}
    for fmt in ("f16fold", "f16pre"):
        blk = WanBlockB200(state, dim, ffn, heads, code_format=fmt)
        cache = (torch.from_numpy(ck8[0]).cuda(), torch.from_numpy(cks[0, ..., 0]).cuda(),
                 torch.from_numpy(cv8[0]).cuda(), torch.from_numpy(cvs[0, ..., 0]).cuda(), cap)
        Xd = X.cuda()
        blk.forward(Xd, blk.modulation_of(time_in.cuda()), cache, at, freq, (frames, h, w), at // (h * w),
                    blk.cross_kv(ctx.cuda()), Buffers(n, dim, ffn, heads, at + n, text, "cuda"))
        outs[fmt] = Xd.cpu() - X
    assert native().device_error() == 0
    assert rel(outs["f16pre"].numpy(), outs["f16fold"].numpy()) <= 1e-3


@pytest.mark.parametrize("case", ["within", "beyond"])
def test_rows_with_widely_spread_group_scales_stay_exact_or_are_refused(case):
    """Rows whose group scales lie far apart: a group of tiny values beside ordinary ones ("within": 2^-20 of the
    row's scale), or beside a group of outliers 256 times larger ("beyond": the tiny group just above the 1e-8
    floor of the scale rule, about 2^33 below the outliers). The prescaled operand holds code * scale * 2^-E_m in
    float16: exact while every group's scale lies within about 2^28 of its row's largest. Within that the values
    equal the folded format's bit for bit and the GEMM the exact per-group promotion (E4M3 codes) within float32
    rounding; beyond it the quantizer refuses the row: device error 8 (wdl_device_error). The E4M3 format, which
    holds every group's scale apart, is exact for the same rows. (A group below the 1e-8 floor quantizes to zeros,
    which every format holds exactly.)"""
    _native = native()
    from wan_dit_lab_b200.quantization import w4a4
    M, K, N = 64, 1024, 256
    x = seeded((M, K), 11)
    for row in (5, 40):
        if case == "within":
            x[row, 128:192] *= 2.0 ** -20
        else:
            x[row, 0:64] *= 256.0
            x[row, 128:192] = x[row, 128:192] / x[row, 128:192].abs().max() * 1e-7  # max |x| = 1e-7 > 1e-8
    x = x.to(torch.bfloat16).cuda()
    W = (seeded((N, K), 12) * 0.02).cuda()
    parts = w4a4.quantize(W, rank=0)
    layer = lambda fmt: w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=fmt)  # noqa: E731
    assert _native.device_error() == 0
    c3, s3 = w4a4.quantize_rows(x, torch.bfloat16, code_format="f16fold")
    assert bool((c3[5, 128:192] != 0).any())  # the tiny group holds nonzero codes
    exact = layer("e4m3")(x).float()
    assert _native.device_error() == 0
    pre, rs = w4a4.quantize_rows(x, torch.bfloat16, code_format="f16pre")
    if case == "within":
        assert _native.device_error() == 0
        assert torch.equal(pre.view(torch.int16), expected_prescaled(c3, s3, rs).view(torch.int16))
        y = layer("f16pre")(x).float()
        assert _native.device_error() == 0
        assert rel(y.cpu().numpy(), exact.cpu().numpy()) <= 2e-4
    else:
        with pytest.raises(RuntimeError, match="prescaled"):
            _native.device_error()
        assert _native.device_error() == 0  # read and cleared
