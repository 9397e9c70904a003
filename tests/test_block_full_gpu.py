"""BASELINE config 3 at full size, in the benchmarked code format (f16pre): one Wan-5B block (dim 3072, 24 heads x
128, FFN 14336 with GELU-tanh, 1392 tokens = 3 latent frames of 16 x 29, 4176 cached FP8 keys of 9 frames, a
512-token prompt projected from 4096 channels) on the B200 kernels against the oracle block (oracle/block.py) on
the same packed W4A4 weights, input, cache and prompt; and the same at config 5's size (704 x 1280: a 2640-token
chunk of 3 frames of 22 x 40 over a full window of 15840 cached keys, attention over 18480 keys).

The north star's tolerances, each stage checked on the GPU's own input to that stage, so that the number is the
stage's own error and not what it inherited:
- every linear (qkv, o, cross q / k / v, cross o, the fused MLP): bf16 relative L2 <= 1e-2 (LINEAR_BAR);
- self-attention: cosine >= 0.999 (COS_BAR) against exact softmax attention over the cache's values, no less
  accurate than the reference's own Sage arithmetic (V re-quantized per channel) measured against the same exact
  result (within 10 %), and within 5e-3 relative L2 of the oracle's emulation of its own P V over the cache's
  per-token V; cross-attention: cosine >= 0.999 against the oracle's Sage arithmetic on the same operands and
  against exact softmax attention;
- 3D RoPE of q and k: max abs error <= 1e-3 (ROPE_BAR); the RMSNorm before it equal in bf16 but for values on
  the other side of a rounding boundary.
The whole chain, the oracle run independently from the same input, on the block's residual update: BLOCK_BAR,
derived from the stage bars: an attention output at cosine 0.999 may be off by sqrt(2 (1 - 0.999)) = 4.5e-2
relative L2, and the linear after it adds up to 1e-2; each of the update's three increments is then within
4.5e-2 + 1e-2 of the oracle's, and so is their sum.

The oracle finishes about 140 query rows (whole 32-token blocks at the start, middle and end of the chunk, the last
one short) after a QKV projection and cache store over every row: oracle.block(rows=...) gives them exactly what
the whole chunk would (tests/test_oracle_block_cpu.py)."""

import math

import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle import fp8 as of
from oracle import rope as orope
from oracle import sage as osage
from test_block_gpu import numpy_parts, random_state

pytestmark = pytest.mark.gpu

LINEAR_BAR, COS_BAR, ROPE_BAR = 1e-2, 0.999, 1e-3
BLOCK_BAR = math.sqrt(2 * (1 - COS_BAR)) + LINEAR_BAR

DIM, HEADS, FFN, TEXT, TEXT_DIM = 3072, 24, 14336, 512, 4096
# (grid of the chunk, cached keys, query rows the oracle finishes): BASELINE config 3 (512 x 928: 1392 tokens over
# 9 cached frames) and a chunk of config 5 (704 x 1280: 2640 tokens over a full window of 18 frames, 18480 keys)
CASES = {"config3": ((3, 16, 29), 4176, np.r_[0:64, 672:704, 1344:1392]),
         "config5": ((3, 22, 40), 15840, np.r_[0:64, 1312:1344, 2624:2640])}


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def bf16(x):
    return ob.bf16(x)


@pytest.fixture(scope="module", params=sorted(CASES))
def run(request):
    """The GPU block's trace and the oracle's, on the case's inputs."""
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.models.block import Buffers, WanBlockB200
    GRID, AT, ROWS = CASES[request.param]
    n = GRID[0] * GRID[1] * GRID[2]
    state = random_state(DIM, FFN, 31)
    blk = WanBlockB200(state, DIM, FFN, HEADS, code_format="f16pre")
    g = torch.Generator().manual_seed(32)
    X = torch.randn(n, DIM, generator=g).to(torch.bfloat16).float()  # bf16 [1, 1392, 3072] ~ N(0, 1)
    time_in = torch.randn(6, DIM, generator=g) * 0.1
    # the prompt: 512 tokens of dim 4096 through a random text embedding (Linear, GELU-tanh, Linear) to 3072
    w0, w2 = torch.randn(DIM, TEXT_DIM, generator=g) * 0.02, torch.randn(DIM, DIM, generator=g) * 0.02
    text = torch.randn(TEXT, TEXT_DIM, generator=g).to(torch.bfloat16).float()
    ctx = (torch.nn.functional.gelu(text @ w0.T, approximate="tanh").to(torch.bfloat16).float() @ w2.T).to(torch.bfloat16)
    cap = AT + n
    ck8, cks = of.quantize_rows(torch.randn(1, cap, HEADS, 128, generator=g).numpy())
    cv8, cvs = of.quantize_rows(torch.randn(1, cap, HEADS, 128, generator=g).numpy())
    freq = orope.table(1024).astype(np.float32)
    start = AT // (GRID[1] * GRID[2])
    cache = (torch.from_numpy(ck8[0]).cuda(), torch.from_numpy(cks[0, ..., 0]).cuda(),
             torch.from_numpy(cv8[0]).cuda(), torch.from_numpy(cvs[0, ..., 0]).cuda(), cap)
    buf = Buffers(n, DIM, FFN, HEADS, cap, TEXT, "cuda")
    mod = blk.modulation_of(time_in.cuda())
    Xd = X.cuda()
    gt = {}
    blk.forward(Xd, mod, cache, AT, torch.from_numpy(freq).cuda(), GRID, start, blk.cross_kv(ctx.cuda()), buf, trace=gt)
    assert _native.device_error() == 0
    cross_k = blk.layers["cross_attn.k"](ctx.cuda()).float().cpu().numpy()
    cross_v = blk.layers["cross_attn.v"](ctx.cuda()).float().cpu().numpy()
    norms = dict(norm_q=blk.norm_q.cpu().numpy(), norm_k=blk.norm_k.cpu().numpy(),
                 cross_norm_q=blk.cross_norm_q.cpu().numpy(), cross_norm_k=blk.cross_norm_k.cpu().numpy(),
                 norm3_w=blk.norm3_w.cpu().numpy(), norm3_b=blk.norm3_b.cpu().numpy())
    parts = numpy_parts(blk.parts)
    ot = {}
    ocache = dict(k=ck8.copy(), ks=cks.copy(), v=cv8.copy(), vs=cvs.copy())
    out_rows = ob.block(X.numpy(), mod.cpu().numpy(), parts, norms, ocache, AT, freq, GRID, start, ctx.float().numpy(),
                        HEADS, trace=ot, rows=ROWS, token_v=True)
    gpu = {k: v.float().cpu().numpy() for k, v in gt.items()}
    gpu["out"] = Xd.cpu().numpy()
    return dict(gpu=gpu, oracle=ot, out_rows=out_rows, X=X.numpy(), mod=mod.cpu().numpy(), parts=parts, norms=norms,
                cache=(ck8, cks, cv8, cvs), cache_gpu=[c.cpu().numpy() for c in cache[:4]], freq=freq, start=start,
                ctx=ctx.float().numpy(), cross_k=cross_k, cross_v=cross_v, n=n, grid=GRID, at=AT, rows=ROWS)


def test_qkv_projection(run):
    got, want = run["gpu"]["qkv"], run["oracle"]["qkv"]  # every row, from the same input
    err = rel(got, want)
    print(f"qkv relative L2 {err:.2e}")
    assert err <= LINEAR_BAR


def test_rms_norm_and_rope_of_q_and_k(run):
    """The fused RMSNorm + RoPE of q and k (one kernel): the norm's output is rounded to bf16 (.type_as of the
    reference's RMSNorm) and scaled by the norm weight before RoPE rotates it. The GPU's result is rotated back in
    float64 to recover its bf16 normalized values (the rotation's own error is far below half a bf16 step); then
    RoPE alone, applied to those values, must match within the north star's 1e-3 max abs error, and the bf16
    normalized values must equal the oracle's but for a float32 sum that lands on the other side of a bf16
    rounding boundary (one bf16 step, at most 0.1 % of the values)."""
    GRID = run["grid"]
    n, qkv = run["n"], run["gpu"]["qkv"]
    c, s_ = orope.angles_for(GRID, run["freq"].astype(np.float64), run["start"], n)
    c, s_ = c[:, None, :], s_[:, None, :]
    for name, cols, w in (("q", slice(0, DIM), run["norms"]["norm_q"]), ("k", slice(DIM, 2 * DIM), run["norms"]["norm_k"])):
        got = run["gpu"][name].reshape(n, HEADS, 128).astype(np.float64)
        back = np.empty_like(got)
        back[..., 0::2] = got[..., 0::2] * c + got[..., 1::2] * s_
        back[..., 1::2] = got[..., 1::2] * c - got[..., 0::2] * s_
        wh = w.reshape(HEADS, 128).astype(np.float64)
        b_gpu = torch.from_numpy((back / wh).astype(np.float32)).to(torch.bfloat16).float().numpy()
        rotated = orope.rope_apply((b_gpu * wh.astype(np.float32)).reshape(1, n, HEADS, 128).astype(np.float32), GRID,
                                   run["freq"], run["start"]).reshape(n, HEADS, 128)
        rope_err = float(np.abs(run["gpu"][name].reshape(n, HEADS, 128) - rotated).max())
        b_oracle = orope.rms_norm(qkv[:, cols], np.ones(DIM, np.float32), round_to="bfloat16").reshape(n, HEADS, 128)
        equal = float((b_gpu == b_oracle).mean())
        # one bf16 step at the larger value's magnitude, plus the float32 noise of rotating back (values of a few
        # units: a few 1e-7), which for a value near zero is worth several of its own bf16 steps
        top = np.maximum(np.abs(b_gpu), np.abs(b_oracle))
        step = np.exp2(np.floor(np.log2(np.maximum(top, 2.0 ** -126))) - 7)
        worst = float((np.abs(b_gpu - b_oracle) / (step + 1e-6)).max())
        print(f"{name}: RoPE max abs error {rope_err:.2e}; RMSNorm bf16 values equal {equal:.5f}, largest "
              f"difference {worst:.2f} (in bf16 steps + 1e-6)")
        assert rope_err <= ROPE_BAR
        assert equal >= 0.999 and worst <= 1.0


def test_fp8_cache_rows_of_the_chunk(run):
    """The chunk's keys and values as the cache stores them (per-(token, head) E4M3 of quantize_rows), from the
    GPU's own K and V: equal bytes and scales but for values within one rounding of a boundary."""
    AT = run["at"]
    n = run["n"]
    K = run["gpu"]["k"].reshape(1, n, HEADS, 128)
    V = run["gpu"]["qkv"][:, 2 * DIM:].reshape(1, n, HEADS, 128)
    for (codes, scales), (gc, gs) in ((of.quantize_rows(K), run["cache_gpu"][0:2]), (of.quantize_rows(V), run["cache_gpu"][2:4])):
        assert (gc[AT:AT + n] == codes[0]).mean() > 0.999
        np.testing.assert_allclose(gs[AT:AT + n], scales[0, ..., 0], rtol=1e-6)


def self_attention_operands(run):
    n = run["n"]
    Q = run["gpu"]["q"].reshape(1, n, HEADS, 128)
    K = run["gpu"]["k"].reshape(1, n, HEADS, 128)
    V = run["gpu"]["qkv"][:, 2 * DIM:].reshape(1, n, HEADS, 128)
    return Q, K, V


def test_self_attention(run):
    AT, ROWS = run["at"], run["rows"]
    ck8, cks, cv8, cvs = run["cache"]
    Q, K, V = self_attention_operands(run)
    got = run["gpu"]["attn"][ROWS]
    # the reference's Sage arithmetic (V re-quantized per channel) and this kernel's (P V over the cache's
    # per-token V, each key's scale folded into P)
    reference = osage.sage_attention(Q, ck8, cks, cv8, cvs, AT, K, V, fp8_p=True, rows=ROWS).reshape(len(ROWS), DIM)
    emulated = osage.sage_attention(Q, ck8, cks, cv8, cvs, AT, K, V, fp8_p=True, rows=ROWS,
                                    token_v=True).reshape(len(ROWS), DIM)
    exact = osage.attention(Q[:, ROWS], osage.load(ck8, cks, K, AT), osage.load(cv8, cvs, V, AT)).reshape(len(ROWS), DIM)
    c_exact = cosine(got, exact)
    print(f"self-attention: cosine {c_exact:.6f} vs exact; relative L2 vs exact {rel(got, exact):.4f} (the "
          f"reference's Sage arithmetic {rel(reference, exact):.4f}); {rel(got, emulated):.2e} vs its own P V emulated")
    assert c_exact >= COS_BAR
    assert rel(got, exact) <= 1.1 * rel(reference, exact)  # no less accurate than the reference's arithmetic
    assert rel(got, emulated) < 5e-3  # the kernel's FP8 P V against its emulation


def test_output_projection_and_gated_residual(run):
    ROWS = run["rows"]
    X, g_a = run["X"][ROWS], run["mod"][2]
    o = bf16(ob.linear(bf16(run["gpu"]["attn"][ROWS]), run["parts"]["self_attn.o"]))
    want = (X + o * g_a).astype(np.float32) - X
    err = rel(run["gpu"]["x_after_self"][ROWS] - X, want)
    print(f"o + gate: relative L2 {err:.2e}")
    assert err <= LINEAR_BAR


def test_cross_attention_projections(run):
    ROWS = run["rows"]
    x3 = bf16(ob.layer_norm(run["gpu"]["x_after_self"][ROWS], w=run["norms"]["norm3_w"], b=run["norms"]["norm3_b"]))
    cq = bf16(ob.linear(x3, run["parts"]["cross_attn.q"]))
    errs = {"cross q": rel(run["gpu"]["cq"][ROWS], cq),
            "cross k": rel(run["cross_k"], bf16(ob.linear(run["ctx"], run["parts"]["cross_attn.k"]))),
            "cross v": rel(run["cross_v"], bf16(ob.linear(run["ctx"], run["parts"]["cross_attn.v"])))}
    print({k: f"{v:.2e}" for k, v in errs.items()})
    assert max(errs.values()) <= LINEAR_BAR


def test_cross_attention(run):
    ROWS = run["rows"]
    m = len(ROWS)
    CQ = orope.rms_norm(run["gpu"]["cq"][ROWS], run["norms"]["cross_norm_q"], round_to="bfloat16").reshape(1, m, HEADS, 128)
    CK = orope.rms_norm(run["cross_k"], run["norms"]["cross_norm_k"], round_to="bfloat16").reshape(1, TEXT, HEADS, 128)
    CV = run["cross_v"].reshape(1, TEXT, HEADS, 128)
    empty = np.zeros((1, 0, HEADS, 128), np.uint8)
    no_scale = np.zeros((1, 0, HEADS, 1), np.float32)
    emulated = osage.sage_attention(CQ, empty, no_scale, empty, no_scale, 0, CK, CV, fp8_p=True).reshape(m, DIM)
    exact = osage.attention(CQ, CK, CV).reshape(m, DIM)
    got = run["gpu"]["cattn"][ROWS]
    c_emu, c_exact = cosine(got, emulated), cosine(got, exact)
    print(f"cross-attention: cosine {c_emu:.6f} vs the oracle's Sage arithmetic, {c_exact:.6f} vs exact")
    assert c_emu >= COS_BAR and c_exact >= COS_BAR


def test_cross_output_projection(run):
    ROWS = run["rows"]
    before = run["gpu"]["x_after_self"][ROWS]
    co = bf16(ob.linear(bf16(run["gpu"]["cattn"][ROWS]), run["parts"]["cross_attn.o"]))
    err = rel(run["gpu"]["x_after_cross"][ROWS] - before, (before + co).astype(np.float32) - before)
    print(f"cross o: relative L2 {err:.2e}")
    assert err <= LINEAR_BAR


def test_feed_forward(run):
    """The fused GELU MLP (FFN-1 with GELU + shift + unsigned INT4 requantization in its epilogue, FFN-2) and the
    gated residual, on the GPU's own input to it."""
    ROWS = run["rows"]
    before = run["gpu"]["x_after_cross"][ROWS]
    sh, sc, g_f = run["mod"][3], run["mod"][4], run["mod"][5]
    x2 = bf16((ob.layer_norm(before) * (np.float32(1) + sc)).astype(np.float32) + sh)
    f, hq, hs = ob.feed_forward(x2, run["parts"])
    err = rel(run["gpu"]["out"][ROWS] - before, (before + f * g_f).astype(np.float32) - before)
    codes_equal = float((run["gpu"]["hcodes"][ROWS] == hq).mean())
    print(f"feed forward: relative L2 {err:.2e}; hidden codes equal {codes_equal:.4f}; "
          f"hidden scales relative L2 {rel(run['gpu']['hscales'][:, ROWS], hs):.2e}")
    assert err <= LINEAR_BAR
    assert codes_equal >= 0.99 and rel(run["gpu"]["hscales"][:, ROWS], hs) <= LINEAR_BAR


def test_block_residual_update_against_the_independent_oracle(run):
    ROWS = run["rows"]
    X = run["X"][ROWS]
    err = rel(run["gpu"]["out"][ROWS] - X, run["out_rows"] - X)
    stages = {k: rel(run["gpu"][k][ROWS], run["oracle"][k]) for k in ("attn", "x_after_self", "cq", "cattn", "x_after_cross")}
    print(f"block residual update relative L2 {err:.4f} (bar {BLOCK_BAR:.4f}); chained stages",
          {k: f"{v:.2e}" for k, v in stages.items()})
    assert err <= BLOCK_BAR
