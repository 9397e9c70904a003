"""The offline rounding options of W4A4 conversion (quantization/w4a4.py: int4_groups(rule="mse"), gptq, and
quantize with them) on the CPU, pinned by the reference's own functions (tests/golden/w4a4_calibration.npz, made by
its int4_groups and gptq, w4a4.py:80-137): codes and scales equal bit for bit. Then the properties the reference's
tests state (tests/test_w4a4.py:144-176): GPTQ's layer output closer to the float layer's than rounding to the
nearest, MSE scales fitting heavy-tailed weights better than the largest-value scales; and quantize's packed
nibbles, scales and shift-corrected bias from those codes."""

from pathlib import Path

import numpy as np
import torch

from oracle import w4a4 as ow

G = np.load(Path(__file__).resolve().parent / "golden" / "w4a4_calibration.npz")


def nearest(R):
    """Rounding to the nearest with the largest-value scales (the "max" rule), in torch on the CPU."""
    N, K = R.shape
    groups = R.view(N, K // 64, 64)
    s = groups.abs().amax(-1).clamp(min=1e-8) / 7
    return torch.round(groups / s[..., None]).clamp(-8, 7).to(torch.int32).view(N, K), s


def dequant(q, s):
    N, K = q.shape
    return (q.view(N, K // 64, 64).float() * s[..., None]).view(N, K)


def test_mse_rule_equals_the_reference():
    from wan_dit_lab_b200.quantization import w4a4
    R = torch.from_numpy(G["R"])
    q, s = w4a4.int4_groups(R, rule="mse")
    np.testing.assert_array_equal(q.numpy(), G["q_mse"])
    np.testing.assert_array_equal(s.numpy(), G["s_mse"])
    # heavy tails: the MSE scales reconstruct the groups better than the largest value's
    err = lambda q, s: float(((R - dequant(q, s)) ** 2).sum())  # noqa: E731
    assert err(q, s) < 0.9 * err(*nearest(R))
    assert q.min() >= -8 and q.max() <= 7


def test_gptq_equals_the_reference():
    from wan_dit_lab_b200.quantization import w4a4
    R, H = torch.from_numpy(G["Rg"]), torch.from_numpy(G["H"])
    q, s = w4a4.gptq(R, H)
    np.testing.assert_array_equal(q.numpy(), G["q_gptq"])
    np.testing.assert_array_equal(s.numpy(), G["s_gptq"])
    assert not q[:, 77].any()  # the idle input channel is rounded from 0
    # || X (R - Q(R))^T ||^2 = tr((R - Q) H (R - Q)^T): GPTQ's output error against rounding to the nearest
    out_err = lambda W: float(torch.einsum("nk,kl,nl->", R - W, H, R - W))  # noqa: E731
    assert out_err(dequant(q, s)) < 0.8 ** 2 * out_err(dequant(*nearest(R)))


def test_quantize_with_offline_rules_packs_their_codes():
    from wan_dit_lab_b200.quantization import w4a4
    g = torch.Generator().manual_seed(3)
    N, K = 64, 256
    W = torch.randn(N, K, generator=g) * 0.02
    b = torch.randn(N, generator=g) * 0.1
    smooth = torch.rand(K, generator=g) + 0.5
    X = torch.randn(512, K, generator=g)
    for kw in (dict(rule="mse"), dict(hessian=X.T @ X)):
        t = w4a4.quantize(W, b, smooth=smooth, rank=0, shift=w4a4.GELU_SHIFT, **kw)
        Ws = W * smooth[None, :]
        q, s = w4a4.int4_groups(Ws, "mse") if "rule" in kw else w4a4.gptq(Ws, X.T @ X / smooth[:, None] / smooth[None, :])
        np.testing.assert_array_equal(ow.unpack_nibbles(t["qweight"].numpy()), q.numpy())
        assert torch.equal(t["wscales"], s.t().to(torch.bfloat16))
        want_b = b - w4a4.GELU_SHIFT * (dequant(q, s) / smooth[None, :]).sum(1)
        assert torch.equal(t["bias"], want_b.to(torch.bfloat16))
        assert t["qweight"].dtype == torch.uint8 and t["qweight"].shape == (N, K // 2)
