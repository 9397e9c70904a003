"""The CPU oracle (oracle/) against golden vectors the reference's own code produced (tests/golden/*.npz, made
by tests/golden/make_golden.py from wan-dit-lab's source). CPU only: this pins the checker the GPU tests use."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import rope as orope
from oracle import sage as osage
from oracle import w4a4 as ow

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / name)


def bf16(bits):
    return torch.from_numpy(np.asarray(bits, np.int16)).view(torch.bfloat16).float().numpy()


def test_int4_groups_matches_reference_bitwise():
    g = load("w4a4_int4_groups.npz")
    q, s = ow.int4_groups(g["R"])
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s, g["scale"])
    np.testing.assert_array_equal(ow.round_to(s, "bfloat16"), bf16(g["scale_bf16"]))
    np.testing.assert_array_equal(ow.round_to(s, "float16"), g["scale_f16"].astype(np.float32))
    qx, sx = ow.int4_groups(bf16(g["x_bf16"]))
    np.testing.assert_array_equal(qx, g["qx"])
    np.testing.assert_array_equal(sx, g["sx"])


def test_nibble_pack_round_trip():
    g = load("w4a4_int4_groups.npz")
    q = g["q"].astype(np.int8)
    packed = ow.pack_nibbles(q)
    assert packed.shape == (q.shape[0], q.shape[1] // 2) and packed.dtype == np.uint8
    np.testing.assert_array_equal(packed[:, 0] & 0xF, q[:, 0].astype(np.uint8) & 0xF)  # low nibble = even k
    np.testing.assert_array_equal(ow.unpack_nibbles(packed), q)
    codes = np.arange(-8, 8, dtype=np.int8)[None, :]
    np.testing.assert_array_equal(ow.unpack_nibbles(ow.pack_nibbles(codes)), codes)


def test_group_partials_are_exact_integers():
    rng = np.random.default_rng(0)
    a = rng.integers(-8, 8, (33, 192)).astype(np.int8)
    w = rng.integers(-8, 8, (40, 192)).astype(np.int8)
    P = ow.group_partials(a, w)
    for g in range(3):
        s = slice(64 * g, 64 * g + 64)
        np.testing.assert_array_equal(P[g], a[:, s].astype(np.int64) @ w[:, s].astype(np.int64).T)
    ext = np.full((1, 64), -8, np.int8)
    assert ow.group_partials(ext, ext)[0, 0, 0] == 4096  # the largest magnitude of a group


def test_fp8_rows_match_reference_bitwise():
    g = load("fp8_rows.npz")
    for name in ("k32", "edge", "mid"):
        for dt in ("float32", "bfloat16", "float16"):
            key = f"{name}_{dt}"
            q, s = of.quantize_rows(g[key + "_x"])
            np.testing.assert_array_equal(q, g[key + "_fp8"], err_msg=key)
            np.testing.assert_array_equal(s, g[key + "_scale"], err_msg=key)


def test_rope_tables_and_apply_match_reference():
    g = load("rope.npz")
    # float64 cos / sin of two libms (numpy here, PyTorch in the reference) may differ in the last bit
    np.testing.assert_allclose(orope.table(64), g["freq64"], rtol=0, atol=4.5e-16)
    grid, start = tuple(g["grid"]), int(g["start"])
    out = orope.rope_apply(g["x32"], grid, g["freq32"], start)
    np.testing.assert_array_equal(out, g["out32_f32table"])  # bitwise: same fp32 operations
    out = orope.rope_apply(g["x32"], grid, g["freq64"], start, out_dtype="float32")
    np.testing.assert_array_equal(out, g["out32_f64table"])
    out = orope.rope_apply(bf16(g["xbf16"]), grid, g["freq32"], start, out_dtype="bfloat16")
    np.testing.assert_array_equal(out, bf16(g["outbf16_f32table"]))


def test_norms_match_reference():
    g = load("norms.npz")
    x = g["x"]
    np.testing.assert_allclose(orope.rms_norm(x, g["rms_weight"]), g["rms_f32"], rtol=2e-6, atol=1e-6)
    np.testing.assert_allclose(orope.rms_norm(bf16(g["xbf16"]), g["rms_weight"], round_to="bfloat16"), g["rms_bf16"],
                               rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(orope.layer_norm(x), g["ln_f32"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(orope.layer_norm(x, weight=g["ln3_weight"], bias=g["ln3_bias"]), g["ln3_f32"],
                               rtol=1e-5, atol=1e-5)


def test_sage_quantizers_match_reference():
    """K int8 within +-1 of the reference (its key mean is summed with float atomics, in any order), scales to
    1e-5; V FP8 bytes >= 99.9 % equal; Q int8 and its scales bitwise (quant_q is plain torch)."""
    g = load("sage_quant.npz")
    at = int(g["at"])
    K = osage.load(g["cache_k"], g["cache_ks"], g["K"], at)
    V = osage.load(g["cache_v"], g["cache_vs"], bf16(g["V"]), at)
    np.testing.assert_allclose(K.sum(axis=1), g["k_sum"][:, :, :], rtol=1e-4, atol=1e-3)
    kq, ks, _ = osage.quant_k(K)
    assert kq.shape == g["k_int8"].shape and ks.shape == g["k_scale"].shape
    assert np.abs(kq.astype(int) - g["k_int8"].astype(int)).max() <= 1
    np.testing.assert_allclose(ks, g["k_scale"], rtol=1e-5)
    v8, vs = osage.quant_v(V)
    np.testing.assert_allclose(vs, g["v_scale"], rtol=1e-6)
    assert v8.shape == g["v_fp8"].shape
    # Triton's CPU interpreter (which made these bytes) does not round float32 to E4M3 to nearest: about 3 % of
    # its bytes sit one E4M3 step away from round-to-nearest (0.4903 -> 0.25, 0.26 -> 0.28125). The
    # round-to-nearest-even contract is pinned by fp8_rows.npz (quantize_rows, the reference's bitwise cache
    # contract) and by the reference's own test against Sage's per_channel_fp8 (tests/test_sage_kv.py:34-56).
    # Here the bytes pin the layout (transposition, padding, the 16-token permutation) and the V scales: >= 96 %
    # of the bytes are equal and every value is within the interpreter's error (at most one binade) of it.
    mine, theirs = of.from_e4m3_bits(v8), of.from_e4m3_bits(g["v_fp8"])
    assert (v8 == g["v_fp8"]).mean() >= 0.96
    assert np.all(np.sign(mine) * np.sign(theirs) >= 0)
    step = np.maximum(np.abs(mine), np.abs(theirs)) / 2 + 2.0 ** -9
    assert np.all(np.abs(mine - theirs) <= step)
    qq, qs = osage.quant_q(g["Q"])
    np.testing.assert_array_equal(qq, g["q_int8"])
    np.testing.assert_array_equal(qs, g["q_scale"])


def test_kv_cache_attention_matches_reference():
    """KVCache(fp8=True).attend: FP8 store, read back, exact attention with the chunk unquantized."""
    g = load("kv_attend.npz")
    per, chunk = int(g["per"]), int(g["chunk"])
    n = per * chunk
    H, D = 2, 128
    cap = 4 * chunk * per + n
    ck = np.zeros((1, cap, H, D), np.uint8)
    cv = np.zeros_like(ck)
    cks = np.zeros((1, cap, H, 1), np.float32)
    cvs = np.zeros_like(cks)
    saved = 0
    for step in range(3):
        at = int(g[f"at{step}"])
        assert at == saved
        q, k, v = g[f"q{step}"], g[f"k{step}"], g[f"v{step}"]
        of.store(ck, cks, cv, cvs, at, k, v)
        keys = np.concatenate([of.from_e4m3_bits(ck[:, :at]) * cks[:, :at], k], axis=1)
        values = np.concatenate([of.from_e4m3_bits(cv[:, :at]) * cvs[:, :at], v], axis=1)
        out = osage.attention(q, keys, values)
        np.testing.assert_allclose(out, g[f"out{step}"], rtol=1e-4, atol=1e-5)
        saved += n


@pytest.mark.parametrize("n", [150, 1392])
def test_sage_dequantized_attention_is_close_to_exact(n):
    """The quantization Sage applies keeps attention close to exact (the reference's tolerance style)."""
    rng = np.random.default_rng(n)
    H, D, at = 2, 128, 200
    Q = rng.standard_normal((1, n, H, D)).astype(np.float32)
    K = (rng.standard_normal((1, n, H, D)) + 0.5).astype(np.float32)
    V = rng.standard_normal((1, n, H, D)).astype(np.float32)
    ck, cks = of.quantize_rows((rng.standard_normal((1, at, H, D)) + 0.5).astype(np.float32))
    cv, cvs = of.quantize_rows(rng.standard_normal((1, at, H, D)).astype(np.float32))
    sage = osage.sage_attention(Q, ck, cks, cv, cvs, at, K, V)
    exact = osage.attention(Q, osage.load(ck, cks, K, at), osage.load(cv, cvs, V, at))
    cos = float((sage * exact).sum() / np.linalg.norm(sage) / np.linalg.norm(exact))
    assert cos >= 0.999


def test_oracle_lowrank_linear_reduces_to_linear():
    """The oracle's low-rank linear without a branch is the plain linear, and its branch is linear in x."""
    rng = np.random.default_rng(5)
    M, K, N, r = 9, 128, 64, 4
    x = ow.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    wq, _, sw = ow.weight(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
    b = rng.standard_normal(N).astype(np.float32)
    y0, _, _ = ow.linear(x, wq, sw, b)
    np.testing.assert_array_equal(ow.linear_lowrank(x, wq, sw, None, None, b), y0)
    down, up = rng.standard_normal((K, r)).astype(np.float32), rng.standard_normal((N, r)).astype(np.float32)
    y = ow.linear_lowrank(x, wq, sw, down, up, b)
    np.testing.assert_allclose(y - y0, (x.astype(np.float64) @ down) @ up.T, rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(ow.lowrank(2 * x, down, up), 2 * ow.lowrank(x, down, up), rtol=1e-6)
