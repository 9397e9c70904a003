"""The SVDQuant low-rank branch and gelu_mlp on the B200 kernels against the CPU oracle (oracle/w4a4.py).

A layer of rank r computes y = INT4 GEMM(x / s) + (x proj_down) proj_up^T + b (reference w4a4.py:141-180,
native/ops/w4a4_ops.cpp:32-38); the down-projection is a thin float32 product and the up-projection is formed in the
GEMM's epilogue (wdl_lowrank: every epilogue thread adds act[m, :] . up[n, :] before the bias), which must equal the
same branch passed as its float32 [M, N] addend (wdl_w4a4_gemm_add) within float32 rounding.
gelu_mlp (w4a4_ops.cpp:44-63) keeps GELU's output for the second layer's branch, which reads it without the shift.
Outputs are bfloat16: relative L2 <= 2e-3 against the float32 oracle (the INT4 codes of the hidden layer may
differ by one where GELU's output lands on a rounding boundary), and a rank-32 layer must be closer to the
unquantized product than the same layer at rank 0."""

import numpy as np
import pytest
import torch

from oracle import w4a4 as ow

pytestmark = pytest.mark.gpu


def native():
    from wan_dit_lab_b200 import _native
    return _native


def seeded(shape, seed, scale=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * scale


def structured_weight(N, K, seed, rank=8, scale=0.02):
    """N(0, scale) plus a strong rank-`rank` part: what the low-rank branch is for (outlier directions)."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(N, K, generator=g) * scale
            + (torch.randn(N, rank, generator=g) @ torch.randn(rank, K, generator=g)) * (4 * scale / rank ** 0.5))


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_layer(parts):
    """The oracle's view of the parts of quantize: integer codes [N, K], stored scales [K/64, N], factors,
    bias and smoothing as float32."""
    f = lambda t: None if t is None else t.float().cpu().numpy()  # noqa: E731
    return dict(codes=ow.unpack_nibbles(parts["qweight"].cpu().numpy()), scales=f(parts["wscales"]),
                down=f(parts["proj_down"]), up=f(parts["proj_up"]), bias=f(parts["bias"]), smooth=f(parts["smooth"]))


@pytest.mark.parametrize("fmt", ["f16pre", "f16fold", "e4m3", "int8"])
@pytest.mark.parametrize("M,N,K", [(300, 768, 1024), (37, 256, 512)])
def test_lowrank_linear_against_oracle(M, N, K, fmt):
    from wan_dit_lab_b200.quantization import w4a4
    x = seeded((M, K), 10).to(torch.bfloat16)
    W = structured_weight(N, K, 11)
    b = seeded((N,), 12, 0.1)
    s = (seeded((K,), 13).abs() + 0.5)
    parts = w4a4.quantize(W.cuda(), b.cuda(), smooth=s.cuda(), rank=32)
    assert parts["proj_down"].shape == (K, 32) and parts["proj_up"].shape == (N, 32)
    layer = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=fmt)
    assert layer.rank == 32
    y = layer(x.cuda()).float().cpu().numpy()
    o = oracle_layer(parts)
    expected = ow.linear_lowrank(x.float().numpy(), o["codes"], o["scales"], o["down"], o["up"], o["bias"],
                                 o["smooth"])
    assert rel(y, expected) <= 2e-3
    exact = x.float().numpy() @ W.numpy().T + b.numpy()[None, :]
    parts0 = w4a4.quantize(W.cuda(), b.cuda(), smooth=s.cuda(), rank=0)
    y0 = w4a4.PreparedW4A4(*(parts0[p] for p in w4a4.PARTS), code_format=fmt)(x.cuda()).float().cpu().numpy()
    assert rel(y, exact) < 0.5 * rel(y0, exact)
    assert native().device_error() == 0


def test_lowrank_linear_module_and_functional_agree():
    from wan_dit_lab_b200.quantization import w4a4
    M, N, K = 130, 512, 768
    x = seeded((2, M, K), 20).to(torch.bfloat16).cuda()
    parts = w4a4.quantize(structured_weight(N, K, 21).cuda(), seeded((N,), 22, 0.1).cuda(), rank=16)
    y_mod = w4a4.PackedW4A4Linear(**parts)(x)
    y_fun = w4a4.linear(x.reshape(-1, K), parts).reshape(2, M, N)
    assert y_mod.shape == (2, M, N)
    assert torch.equal(y_mod, y_fun)


def gelu_mlp_parts(K, H, N2, rank, seed):
    from wan_dit_lab_b200.quantization import w4a4
    W1, W2 = structured_weight(H, K, seed), structured_weight(N2, H, seed + 1)
    b1, b2 = seeded((H,), seed + 2, 0.1), seeded((N2,), seed + 3, 0.1)
    s2 = seeded((H,), seed + 4).abs() + 0.5
    t1 = w4a4.quantize(W1.cuda(), b1.cuda(), rank=rank)
    t2 = w4a4.quantize(W2.cuda(), b2.cuda(), smooth=s2.cuda(), rank=rank, shift=w4a4.GELU_SHIFT)
    return (W1, b1, W2, b2), t1, t2


@pytest.mark.parametrize("rank", [0, 32])
@pytest.mark.parametrize("M", [300, 37])
def test_gelu_mlp_against_oracle(M, rank):
    from wan_dit_lab_b200.quantization import w4a4
    K, H, N2 = 512, 1024, 256
    (W1, b1, W2, b2), t1, t2 = gelu_mlp_parts(K, H, N2, rank, 30)
    x = seeded((M, K), 35).to(torch.bfloat16)
    y = w4a4.gelu_mlp(x.cuda(), t1, t2).float().cpu().numpy()
    o1, o2 = oracle_layer(t1), oracle_layer(t2)
    if not rank:
        o1["down"] = o1["up"] = o2["down"] = o2["up"] = None
    expected = ow.gelu_mlp(x.float().numpy(), o1, o2)
    assert rel(y, expected) <= 2e-3
    h = x.float().numpy() @ W1.numpy().T + b1.numpy()[None, :]
    exact = ow.gelu_tanh(h) @ W2.numpy().T + b2.numpy()[None, :]
    assert rel(y, exact) < 0.4
    y_mod = w4a4.PackedW4A4GeluMLP(t1, t2)(x.cuda().reshape(1, M, K))
    assert torch.equal(y_mod.reshape(M, N2).float().cpu(), torch.from_numpy(y))
    assert native().device_error() == 0


def test_gelu_mlp_lowrank_improves_on_rank0():
    from wan_dit_lab_b200.quantization import w4a4
    K, H, N2, M = 512, 1024, 256, 200
    x = seeded((M, K), 45).to(torch.bfloat16)
    errs = []
    for rank in (0, 32):
        (W1, b1, W2, b2), t1, t2 = gelu_mlp_parts(K, H, N2, rank, 40)
        y = w4a4.gelu_mlp(x.cuda(), t1, t2).float().cpu().numpy()
        h = x.float().numpy() @ W1.numpy().T + b1.numpy()[None, :]
        errs.append(rel(y, ow.gelu_tanh(h) @ W2.numpy().T + b2.numpy()[None, :]))
    assert errs[1] < 0.5 * errs[0]


def test_gemm_add_rejects_misaligned_addend():
    """The addend is read as float32 rows: ld_add below N is an argument error before any launch."""
    _native = native()
    M, N, K = 64, 256, 128
    a = torch.zeros(M, K, dtype=torch.int8, device="cuda")
    sa = torch.ones(K // 64, M, device="cuda")
    w = torch.zeros(N, K, dtype=torch.int8, device="cuda")
    sw = torch.ones(K // 64, N, device="cuda")
    add = torch.zeros(M, N, device="cuda")
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    st = _native.lib().wdl_w4a4_gemm_add(a.data_ptr(), sa.data_ptr(), w.data_ptr(), sw.data_ptr(), 0, None,
                                          add.data_ptr(), N - 1, M, N, K, y.data_ptr(), N, _native.stream())
    assert st == _native.ERR_ARGUMENT
    st = _native.lib().wdl_w4a4_gemm_add(a.data_ptr(), sa.data_ptr(), w.data_ptr(), sw.data_ptr(), 0, None,
                                          add.data_ptr(), N, M, N, K, y.data_ptr(), N, _native.stream())
    assert st == 0
    torch.cuda.synchronize()
    assert float(y.float().abs().max()) == 0.0


@pytest.mark.parametrize("fmt", ["f16pre", "f16fold", "e4m3", "int8"])
@pytest.mark.parametrize("rank", [6, 32])
def test_epilogue_branch_equals_its_addend(fmt, rank):
    """The branch formed in the GEMM epilogue against the same branch passed as a float32 [M, N] addend, in each
    output mode: the float32 product (wdl_w4a4_gemm_f32*) within float32 rounding of the sum (the epilogue adds
    one rank after the other onto the product, the addend is added once), bf16 outputs and the gated residual
    update at most one bf16 step apart where the two sums straddle a rounding boundary. Rank 6 runs padded to 8
    with zero columns."""
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    lib, st = _native.lib(), _native.stream()
    M, N, K = 300, 768, 1024
    x = seeded((M, K), 50).to(torch.bfloat16).cuda()
    parts = w4a4.quantize(structured_weight(N, K, 51).cuda(), seeded((N,), 52, 0.1).cuda(),
                          smooth=(seeded((K,), 53).abs() + 0.5).cuda(), rank=rank)
    layer = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=fmt)
    assert layer.rank == rank and layer.up.shape[1] == -(-rank // 4) * 4
    act = layer.lowrank_act(x)
    add = (act.double() @ layer.up.double().t()).float().contiguous()
    work = torch.empty(lib.wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device="cuda")
    codes, scales = layer.quantize_input(x, work)
    args = (codes.data_ptr(), scales.data_ptr(), layer.codes.data_ptr(), layer.scales.data_ptr(), layer.code_format,
            _native.ptr(layer.bias))
    f_lr, f_add = (torch.empty(M, N, device="cuda") for _ in range(2))
    _native.check(lib.wdl_w4a4_gemm_f32_lowrank(*args, layer.lowrank_arg(act), M, N, K, f_lr.data_ptr(), N, st))
    _native.check(lib.wdl_w4a4_gemm_f32(*args, add.data_ptr(), N, M, N, K, f_add.data_ptr(), N, st))
    b_lr, b_add = (torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    _native.check(lib.wdl_w4a4_gemm_lowrank(*args, layer.lowrank_arg(act), M, N, K, b_lr.data_ptr(), N, st))
    _native.check(lib.wdl_w4a4_gemm_add(*args, add.data_ptr(), N, M, N, K, b_add.data_ptr(), N, st))
    residual = seeded((M, N), 54).cuda()
    gate = (seeded((N,), 55, 0.5)).cuda()
    r_lr, r_add = residual.clone(), residual.clone()
    _native.check(lib.wdl_w4a4_gemm_residual_lowrank(*args, layer.lowrank_arg(act), gate.data_ptr(),
                                                     r_lr.data_ptr(), N, M, N, K, r_lr.data_ptr(), N, st))
    _native.check(lib.wdl_w4a4_gemm_residual_add(*args, add.data_ptr(), N, gate.data_ptr(), r_add.data_ptr(), N, M,
                                                 N, K, r_add.data_ptr(), N, st))
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    branch = float(add.abs().max())
    assert branch > 0.1 * float(f_add.abs().max())  # the branch carries a real share of the output
    tol = 1e-5 * float(f_add.abs().max())  # the two float32 sums: a few ulps of the accumulator apart
    assert float((f_lr - f_add).abs().max()) <= tol
    # bf16 outputs: the sums' difference, plus one bf16 step where they straddle a rounding boundary
    step = lambda a, b: torch.maximum(a.float().abs(), b.float().abs()) * 2.0 ** -7 + tol  # noqa: E731
    assert bool(((b_lr.float() - b_add.float()).abs() <= step(b_lr, b_add)).all())
    assert float((b_lr == b_add).float().mean()) > 0.99
    # the update x + o gate: o as above times the gate, the float32 sum with x rounded once more (|x| < 8)
    o_lr, o_add = r_lr - residual, r_add - residual
    assert bool(((r_lr - r_add).abs() <= step(o_lr, o_add) + 2e-6).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("M,K,rank", [(37, 512, 8), (300, 3072, 32), (300, 14336, 32), (64, 1024, 36)])
def test_lowrank_down_projection(M, K, rank, dtype):
    """wdl_lowrank_down (x proj_down, K split over a cluster of 1 to 8 CTAs whose sums are added in rank order)
    against the float64 product: within float32 rounding of the sum, and bit for bit the same on a second call."""
    _native = native()
    lib, st = _native.lib(), _native.stream()
    x = seeded((M, K), 60).to(dtype).cuda()
    down = seeded((K, rank), 61, 0.05).cuda()
    acts = []
    for _ in range(2):
        act = torch.full((M, rank), float("nan"), device="cuda")
        _native.check(lib.wdl_lowrank_down(x.data_ptr(), _native.DTYPE_CODE[dtype], K, M, K, down.data_ptr(), rank,
                                           act.data_ptr(), rank, st))
        acts.append(act)
    torch.cuda.synchronize()
    want = x.double() @ down.double()
    err = float((acts[0].double() - want).abs().max() / want.abs().max())
    assert err <= 2e-6, err
    assert torch.equal(acts[0], acts[1])
