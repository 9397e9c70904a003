"""The SVDQuant low-rank branch and gelu_mlp on the B200 kernels against the CPU oracle (oracle/w4a4.py).

A layer of rank r computes y = INT4 GEMM(x / s) + (x proj_down) proj_up^T + b (reference w4a4.py:141-180,
native/ops/w4a4_ops.cpp:32-38); the branch's [M, N] product enters the GEMM's epilogue (wdl_w4a4_gemm_add).
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


@pytest.mark.parametrize("fmt", ["f16fold", "e4m3", "int8"])
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
