"""The live::* operators (kernels/operators.py) without a GPU: load() registers live::w4a4_linear,
live::w4a4_gelu_mlp and live::sage_sm89 once and returns torch.ops.live, as the reference's operators.load does
(kernels/operators.py:19-25); their fake implementations give the shapes of the reference's Meta kernels
(native/ops/w4a4_ops.cpp:65-75, native/ops/sage_ops.cpp:21-24) on meta tensors and under FakeTensorMode; Sage's
operand layouts (the reference's quantizers, tests/golden/sage_quant.npz) are rearranged into the kernel's
exactly; malformed Sage operands are refused before any launch."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sage as osage

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def operators():
    from wan_dit_lab_b200.kernels import operators
    return operators


def w4a4_parts(N, K, device, rank=0):
    return [torch.empty(N, K // 2, dtype=torch.uint8, device=device),
            torch.empty(K // 64, N, dtype=torch.bfloat16, device=device),
            torch.empty(K, rank, dtype=torch.bfloat16, device=device),
            torch.empty(N, rank, dtype=torch.bfloat16, device=device),
            torch.empty(K, dtype=torch.bfloat16, device=device), torch.empty(N, dtype=torch.bfloat16, device=device)]


def test_load_registers_once_with_fake_shapes(operators):
    from torch._subclasses.fake_tensor import FakeTensorMode
    ops = operators.load()
    assert ops is torch.ops.live and operators.load() is ops
    x = torch.empty(5, 256, dtype=torch.bfloat16, device="meta")
    y = ops.w4a4_linear(x, *w4a4_parts(384, 256, "meta", 16))
    assert y.shape == (5, 384) and y.dtype == torch.bfloat16
    y = ops.w4a4_gelu_mlp(x, *w4a4_parts(1024, 256, "meta"), *w4a4_parts(256, 1024, "meta"))
    assert y.shape == (5, 256)
    with FakeTensorMode():
        q = torch.empty(1, 150, 2, 128, dtype=torch.int8, device="cuda")
        k = torch.empty(1, 350, 2, 128, dtype=torch.int8, device="cuda")
        v = torch.empty(1, 128, 2, 384, dtype=torch.float8_e4m3fn, device="cuda")
        o = ops.sage_sm89(q, k, v, torch.empty(1, 2, 64, device="cuda"), torch.empty(1, 2, 24, device="cuda"),
                          torch.empty(1, 2, 128, device="cuda"), 0.088)
        assert o.shape == (1, 150, 2, 128) and o.dtype == torch.bfloat16 and o.device.type == "cuda"


def test_cpu_tensors_are_refused(operators):
    ops = operators.load()
    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        ops.w4a4_linear(x, *w4a4_parts(128, 128, "cpu"))


def test_sage_layouts_rearranged_exactly(operators):
    g = np.load(GOLDEN / "sage_quant.npz")
    q, qs, k, ks, v, vs = (torch.from_numpy(g[name]) for name in ("q_int8", "q_scale", "k_int8", "k_scale", "v_fp8",
                                                                   "v_scale"))
    _, n, H, D = q.shape
    L = k.shape[1]
    operators._check_sage(q, k, v.view(torch.float8_e4m3fn), qs, ks, vs)
    qi, qs2, ki, ks2, vf, vs2 = operators.sage_operands(q[0], k[0], v[0].view(torch.float8_e4m3fn), qs[0], ks[0],
                                                        vs[0])
    npad, lpad = -(-n // 128) * 128, -(-L // 128) * 128
    assert qi.shape == (H, npad, D) and ki.shape == (H, lpad, D) and vf.shape == (H, D, lpad)
    assert qs2.shape == (H, npad // 4) and ks2.shape == (H, lpad // 16)
    np.testing.assert_array_equal(qi[:, :n].numpy(), g["q_int8"][0].transpose(1, 0, 2))
    np.testing.assert_array_equal(ki[:, :L].numpy(), g["k_int8"][0].transpose(1, 0, 2))
    assert not qi[:, n:].any() and not ki[:, L:].any() and not vf[:, :, L:].any()
    np.testing.assert_array_equal(qs2.numpy(), g["q_scale"][0])
    np.testing.assert_array_equal(ks2[:, :ks.shape[-1]].numpy(), g["k_scale"][0])
    # V in key order: the oracle's inverse of the reference's 16-key permutation
    np.testing.assert_array_equal(vf[:, :, :L].numpy(), osage.unpermute_v(g["v_fp8"], L)[0].transpose(1, 2, 0))
    np.testing.assert_array_equal(vs2.numpy(), g["v_scale"][0])


def test_malformed_sage_operands_refused(operators):
    q = torch.zeros(1, 150, 2, 128, dtype=torch.int8)
    k = torch.zeros(1, 350, 2, 128, dtype=torch.int8)
    v = torch.zeros(1, 128, 2, 384, dtype=torch.float8_e4m3fn)
    qs, ks, vs = torch.zeros(1, 2, 64), torch.zeros(1, 2, 24), torch.zeros(1, 2, 128)
    operators._check_sage(q, k, v, qs, ks, vs)
    with pytest.raises(TypeError):
        operators._check_sage(q.float(), k, v, qs, ks, vs)
    with pytest.raises(ValueError, match="v"):
        operators._check_sage(q, k, v[..., :320], qs, ks, vs)
    with pytest.raises(ValueError, match="q_scale"):
        operators._check_sage(q, k, v, qs[..., :8], ks, vs)
    with pytest.raises(ValueError, match="v_scale"):
        operators._check_sage(q, k, v, qs, ks, vs[..., :64])
