"""The live::* operators on the B200 (kernels/operators.py), as the reference's call sites use them
(quantization/w4a4.py:210-215, kernels/sage_kv.py:175-176): live::w4a4_linear and live::w4a4_gelu_mlp return what
w4a4_linear / w4a4_gelu_mlp return, bit for bit; live::sage_sm89 over Sage's operand layouts equals attention
over the same operands in the kernel's own layouts bit for bit, and, over the operands the reference's own
quantizers wrote (tests/golden/sage_quant.npz), stays within 5e-3 of the oracle's FP8-P emulation over them (the
bar of the attention kernel's own test); torch.library.opcheck accepts the W4A4 operators' schemas and fake
implementations, and sage_sm89's fake implementation gives its real output's shape, dtype and device."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import sage as osage

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_w4a4_operators_equal_the_module_functions():
    from wan_dit_lab_b200.kernels import operators
    from wan_dit_lab_b200.quantization import w4a4
    ops = operators.load()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(300, 512, generator=g).to(torch.bfloat16).cuda()
    l1 = w4a4.quantize((torch.randn(1024, 512, generator=g) * 0.02).cuda(), (torch.randn(1024, generator=g) * 0.1).cuda(),
                       rank=16)
    l2 = w4a4.quantize((torch.randn(512, 1024, generator=g) * 0.02).cuda(), (torch.randn(512, generator=g) * 0.1).cuda(),
                       rank=16, shift=w4a4.GELU_SHIFT)
    p1, p2 = [l1[p] for p in w4a4.PARTS], [l2[p] for p in w4a4.PARTS]
    assert torch.equal(ops.w4a4_linear(x, *p1), w4a4.w4a4_linear(x, *p1))
    assert torch.equal(ops.w4a4_gelu_mlp(x, *p1, *p2), w4a4.w4a4_gelu_mlp(x, *p1, *p2))
    torch.library.opcheck(ops.w4a4_linear.default, (x, *p1), test_utils=("test_schema", "test_faketensor"))
    torch.library.opcheck(ops.w4a4_gelu_mlp.default, (x, *p1, *p2), test_utils=("test_schema", "test_faketensor"))


def to_sage_layouts(ops, n, L):
    """The kernel's operands (sage_kv.prepare) in Sage's layouts, as the reference's quantizers write them."""
    from wan_dit_lab_b200.kernels.operators import _V_POSITION
    H = ops["q_i8"].shape[0]
    q = ops["q_i8"][:, :n].transpose(0, 1)[None].contiguous()
    k = ops["k_i8"][:, :L].transpose(0, 1)[None].contiguous()
    padded = -(-L // 64) * 64
    natural = ops["v_f8"][:, :, :padded].reshape(H, 128, padded // 16, 16)
    v = torch.empty_like(natural)
    v[..., torch.tensor(_V_POSITION, device=natural.device)] = natural
    v = v.reshape(H, 128, padded).permute(1, 0, 2)[None].contiguous().view(torch.float8_e4m3fn)
    q_scale = ops["q_scale"][None].contiguous()
    k_scale = ops["k_scale"][:, :padded // 16][None].contiguous()
    return q, k, v, q_scale, k_scale, ops["v_scale"][None].contiguous()


@pytest.mark.parametrize("at,n,H", [(200, 150, 2), (4176, 1392, 4)])
def test_sage_operator_equals_the_kernel_on_its_own_layouts(at, n, H):
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.kernels import operators, sage_kv
    g = torch.Generator().manual_seed(at + n)
    total = at + n + 64
    ck, cks = of.quantize_rows((torch.randn(1, total, H, 128, generator=g) + 0.5).numpy())
    cv, cvs = of.quantize_rows((torch.randn(1, total, H, 128, generator=g) * 0.7).numpy())
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    ck, cv = dev(ck).view(torch.float8_e4m3fn), dev(cv).view(torch.float8_e4m3fn)
    cks, cvs = dev(cks), dev(cvs)
    K = (torch.randn(1, n, H, 128, generator=g) + 0.5).cuda()
    V = torch.randn(1, n, H, 128, generator=g).to(torch.bfloat16).cuda()
    Q = torch.randn(1, n, H, 128, generator=g).cuda()
    prepared = sage_kv.prepare(Q, ck, cks, cv, cvs, at, K, V)
    # the kernel on the prepared per-channel operands in this library's layouts (wdl_sage_attention)
    want = torch.empty(1, n, H, 128, dtype=torch.bfloat16, device="cuda")
    lib = _native.lib()
    _native.check(lib.wdl_sage_attention(*(prepared[x].data_ptr() for x in ("q_i8", "q_scale", "k_i8", "k_scale",
                                                                            "v_f8", "v_scale")),
                                         n, at + n, H, 128 ** -0.5, want.data_ptr(), H * 128, _native.stream()))
    args = to_sage_layouts(prepared, n, at + n)
    got = operators.load().sage_sm89(*args, 128 ** -0.5)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert got.shape == want.shape and torch.equal(got, want)
    # the fake implementation gives the real output's metadata (opcheck's schema test cannot compare float8 inputs)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode() as mode:
        fake = operators.load().sage_sm89(*(mode.from_tensor(a) for a in args), 128 ** -0.5)
    assert fake.shape == got.shape and fake.dtype == got.dtype and fake.device == got.device


def test_sage_operator_on_the_reference_quantizers_operands():
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.kernels import operators
    gold = np.load(GOLDEN / "sage_quant.npz")
    names = ("q_int8", "k_int8", "v_fp8", "q_scale", "k_scale", "v_scale")
    t = {name: torch.from_numpy(gold[name]).cuda() for name in names}
    t["v_fp8"] = t["v_fp8"].view(torch.float8_e4m3fn)
    out = operators.load().sage_sm89(*(t[name] for name in names), 128 ** -0.5).float().cpu().numpy()
    assert _native.device_error() == 0
    L = gold["k_int8"].shape[1]
    q = osage.dequant_q(gold["q_int8"], gold["q_scale"])
    k = osage.dequant_k(gold["k_int8"], gold["k_scale"])
    v_codes = of.from_e4m3_bits(osage.unpermute_v(gold["v_fp8"], L))
    emulated = osage.attention_fp8_p(q, k, v_codes, gold["v_scale"])
    assert float(np.linalg.norm(out - emulated) / np.linalg.norm(emulated)) < 5e-3
