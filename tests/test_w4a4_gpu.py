"""W4A4 on the B200 kernels against the CPU oracle (oracle/w4a4.py), through the C ABI.

Bit-exact: activation/weight INT4 codes, their stored scales, the packed nibbles, the unpacked weight, and the
integer group partials read from the tensor-core accumulators. Within tolerance: the bf16 outputs (relative L2
<= 1e-2 is the stated bar for linears; the float32 oracle rounded to bf16 is matched far tighter, <= 2e-3)."""

import numpy as np
import pytest
import torch

from oracle import fp8 as of
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


@pytest.mark.parametrize("M,K,dtype,smooth", [(300, 1024, torch.bfloat16, False), (37, 256, torch.float32, False),
                                              (129, 3072, torch.bfloat16, True), (1, 64, torch.bfloat16, False)])
@pytest.mark.parametrize("scale_dtype", [torch.bfloat16, torch.float16])
def test_quantize_rows_bitwise(M, K, dtype, smooth, scale_dtype):
    from wan_dit_lab_b200.quantization import w4a4
    x = seeded((M, K), 11, outliers=0.01).to(dtype)
    s = (torch.rand(K, generator=torch.Generator().manual_seed(3)) + 0.5).to(torch.bfloat16) if smooth else None
    codes, scales, packed = w4a4.quantize_rows(x.cuda(), scale_dtype, None if s is None else s.cuda(), packed=True)
    xq, sx = ow.int4_groups(x.float().numpy(), None if s is None else s.float().numpy())
    np.testing.assert_array_equal(codes.cpu().numpy(), xq)
    e4m3, _ = w4a4.quantize_rows(x.cuda(), scale_dtype, None if s is None else s.cuda(), code_format="e4m3")
    np.testing.assert_array_equal(e4m3.cpu().numpy(), of.to_e4m3_bits(xq.astype(np.float32)))
    np.testing.assert_array_equal(scales.cpu().numpy(), ow.round_to(sx, str(scale_dtype).split(".")[1]).T)
    np.testing.assert_array_equal(packed.cpu().numpy(), ow.pack_nibbles(xq))


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
def test_unpack_weight_bitwise(fmt):
    _native = native()
    N, K = 512, 384
    g = torch.Generator().manual_seed(5)
    packed = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    ws = (torch.rand(K // 64, N, generator=g) * 0.01).to(torch.float16)
    codes = torch.empty(N, K, dtype=torch.uint8, device="cuda")
    scales = torch.empty(K // 64, N, dtype=torch.float32, device="cuda")
    pc, wc = packed.cuda(), ws.cuda()
    _native.check(_native.lib().wdl_w4a4_unpack_weight(pc.data_ptr(), wc.data_ptr(), _native.F16, N, K,
                                                       FMT[fmt], codes.data_ptr(), scales.data_ptr(), _native.stream()))
    np.testing.assert_array_equal(codes.cpu().numpy(), as_bytes(ow.unpack_nibbles(packed.numpy()), fmt))
    np.testing.assert_array_equal(scales.cpu().numpy(), ws.float().numpy())


FMT = {"int8": 0, "e4m3": 1}


def as_bytes(codes, fmt):
    """Integer codes as the GEMM's operand bytes."""
    codes = np.asarray(codes)
    return codes.astype(np.int8).view(np.uint8) if fmt == "int8" else of.to_e4m3_bits(codes.astype(np.float32))


def dev(codes, fmt):
    return torch.from_numpy(np.ascontiguousarray(as_bytes(codes.numpy(), fmt))).cuda()


def random_codes(shape, seed, unsigned=False):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0 if unsigned else -8, 16 if unsigned else 8, shape, generator=g, dtype=torch.int8)


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
@pytest.mark.parametrize("M,N,K,groups,unsigned", [(300, 512, 512, (0, 3, 7), False), (1392, 9216, 3072, (0, 21, 47), False),
                                                   (129, 256, 1024, (0, 15), True)])
def test_group_partials_bit_exact(M, N, K, groups, unsigned, fmt):
    """The tensor cores' group accumulators, one group at a time, equal the exact integer sums (int32 from
    kind::i8; float32 holding exact integers from kind::f8f6f4, read back as int32). Unsigned activation codes
    [0, 15] (the fused MLP's hidden layer) only in the E4M3 format."""
    if unsigned and fmt == "int8":
        pytest.skip("int8 codes are signed only")
    _native = native()
    a, w = random_codes((M, K), 1, unsigned), random_codes((N, K), 2)
    sa = torch.ones(K // 64, M)
    sw = torch.ones(K // 64, N)
    ac, wc, sac, swc = dev(a, fmt), dev(w, fmt), sa.cuda(), sw.cuda()
    out = torch.empty(M, N, dtype=torch.int32, device="cuda")
    for group in groups:
        _native.check(_native.lib().wdl_w4a4_gemm_group_partials(
            ac.data_ptr(), sac.data_ptr(), wc.data_ptr(), swc.data_ptr(), FMT[fmt], M, N, K, group,
            out.data_ptr(), N, _native.stream()))
        expected = ow.group_partials(a.numpy(), w.numpy(), [group])[0]
        np.testing.assert_array_equal(out.cpu().numpy(), expected)
    assert native().device_error() == 0


@pytest.mark.parametrize("fmt", ["int8", "e4m3"])
@pytest.mark.parametrize("M,N,K", [(300, 768, 1024), (1, 256, 128), (1392, 9216, 3072), (200, 3072, 14336)])
def test_gemm_matches_oracle(M, N, K, fmt):
    _native = native()
    a, w = random_codes((M, K), 3), random_codes((N, K), 4)
    g = torch.Generator().manual_seed(6)
    sa = ow.round_to((torch.rand(K // 64, M, generator=g) * 0.5 + 0.01).numpy(), "bfloat16")
    sw = ow.round_to((torch.rand(K // 64, N, generator=g) * 0.01 + 1e-4).numpy(), "bfloat16")
    bias = (torch.randn(N, generator=g) * 0.1).numpy()
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ac, wc = dev(a, fmt), dev(w, fmt)
    sac, swc, bc = (torch.from_numpy(t).cuda() for t in (sa, sw, bias))
    _native.check(_native.lib().wdl_w4a4_gemm(ac.data_ptr(), sac.data_ptr(), wc.data_ptr(), swc.data_ptr(), FMT[fmt],
                                               bc.data_ptr(), M, N, K, y.data_ptr(), N, _native.stream()))
    expected = ow.gemm(a.numpy(), sa, w.numpy(), sw, bias)
    got = y.float().cpu().numpy()
    assert rel(got, expected) <= 2e-3
    assert rel(got, ow.round_to(expected, "bfloat16")) <= 1e-3
    assert native().device_error() == 0


def test_residual_epilogue_matches_oracle():
    _native = native()
    M, N, K = 257, 512, 768
    a, w = random_codes((M, K), 7), random_codes((N, K), 8)
    g = torch.Generator().manual_seed(9)
    sa = ow.round_to((torch.rand(K // 64, M, generator=g) * 0.5 + 0.01).numpy(), "bfloat16")
    sw = ow.round_to((torch.rand(K // 64, N, generator=g) * 0.01 + 1e-4).numpy(), "bfloat16")
    bias = (torch.randn(N, generator=g) * 0.1).numpy()
    gate = torch.randn(N, generator=g).numpy()
    res = torch.randn(M, N, generator=g).numpy()
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    t = [torch.from_numpy(np.ascontiguousarray(v)).cuda() for v in (sa, sw, bias, gate, res)]
    ac, wc = dev(a, "e4m3"), dev(w, "e4m3")
    for use_gate in (True, False):
        _native.check(_native.lib().wdl_w4a4_gemm_residual(
            ac.data_ptr(), t[0].data_ptr(), wc.data_ptr(), t[1].data_ptr(), 1, t[2].data_ptr(),
            t[3].data_ptr() if use_gate else None, t[4].data_ptr(), N, M, N, K, out.data_ptr(), N, _native.stream()))
        o = ow.round_to(ow.gemm(a.numpy(), sa, w.numpy(), sw, bias), "bfloat16")
        expected = res + o * gate[None, :] if use_gate else res + o
        assert rel(out.cpu().numpy(), expected) <= 1e-4


@pytest.mark.parametrize("fmt", ["e4m3", "int8"])
@pytest.mark.parametrize("M", [1392, 300, 37])
def test_packed_linear_config1_against_oracle(M, fmt):
    """BASELINE config 1 (at M = 1392): X [M, 3072] bf16 N(0,1) with 1% outlier channels x20, W [9216, 3072]
    N(0, 0.02), symmetric INT4 groups of 64 with float16 scales, no bias."""
    from wan_dit_lab_b200.quantization import w4a4
    K, N = 3072, 9216
    x = seeded((M, K), 0, outliers=0.01).to(torch.bfloat16)
    W = seeded((N, K), 1, scale=0.02)
    parts = w4a4.quantize(W.cuda(), rank=0, scale_dtype=torch.float16)
    layer = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=fmt)
    y = layer(x.cuda()).float().cpu().numpy()
    wq, _, sw = ow.weight(W.numpy(), "float16")
    np.testing.assert_array_equal(parts["qweight"].cpu().numpy(), ow.pack_nibbles(wq))
    np.testing.assert_array_equal(parts["wscales"].float().cpu().numpy(), sw)
    expected, _, _ = ow.linear(x.float().numpy(), wq, sw, None, None, "float16")
    assert rel(y, expected) <= 2e-3
    exact = x.float().numpy() @ W.numpy().T  # the unquantized product: W4A4 error is INT4 noise, not kernel error
    assert rel(y, exact) < 0.25
    assert native().device_error() == 0


def test_invalid_arguments_raise_before_launch():
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    x = torch.randn(8, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        w4a4.quantize_rows(x)  # K not a multiple of 64
    a = torch.zeros(8, 128, dtype=torch.int8, device="cuda")
    s = torch.ones(2, 8, device="cuda")
    y = torch.empty(8, 200, dtype=torch.bfloat16, device="cuda")
    st = _native.lib().wdl_w4a4_gemm(a.data_ptr(), s.data_ptr(), a.data_ptr(), s.data_ptr(), 1, None, 8, 200, 128,
                                    y.data_ptr(), 200, _native.stream())
    assert st == _native.ERR_ARGUMENT and b"256" in _native.lib().wdl_last_error()


def test_prepared_layers_follow_the_weight_objects_not_their_addresses():
    """w4a4_linear keeps each layer's device layout on its qweight tensor: a weight freed and another allocated in
    its place (very likely at the same address) gets its own layout, an in-place change of a part is seen, and
    many layers each keep theirs (no shared table to overflow)."""
    from wan_dit_lab_b200.quantization import w4a4
    g = torch.Generator().manual_seed(31)
    M, K, N = 256, 512, 512
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()

    def parts(seed):
        gg = torch.Generator().manual_seed(seed)
        return w4a4.quantize((torch.randn(N, K, generator=gg) * 0.02).cuda(), rank=0)

    def fresh(p):
        return w4a4.PackedW4A4Linear(**{k: v.clone() for k, v in p.items()})(x)

    a = parts(1)
    ya = w4a4.linear(x, a)
    assert torch.equal(ya, fresh(a))
    address = a["qweight"].data_ptr()
    del a
    b = parts(2)
    yb = w4a4.linear(x, b)
    assert torch.equal(yb, fresh(b)) and not torch.equal(yb, ya)
    print("same address reused:", b["qweight"].data_ptr() == address)
    b["wscales"].mul_(2)  # in place: the layout must be remade
    assert torch.equal(w4a4.linear(x, b), fresh(b))
    many = [parts(100 + i) for i in range(300)]  # more layers than one model holds, each its own layout
    for p in many[:3] + many[-3:]:
        assert torch.equal(w4a4.linear(x, p), fresh(p))
    assert all(getattr(p["qweight"], "_wdl_prepared", None) is not None for p in many[:3] + many[-3:])
