"""The oracle block computed for a subset of query rows (whole aligned blocks of 32 tokens, oracle.block.rows)
gives those rows exactly what the whole-chunk oracle gives them, bit for bit: the full-size GPU parity tests
(1392 tokens) compare the B200 block with the oracle on such a subset, which finishes in
seconds on the CPU. Also: the oracle GEMM equals the plain sum over its exact integer group partials."""

import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle import fp8 as of
from oracle import rope as orope
from oracle import w4a4 as ow


def random_parts(dim, ffn, seed):
    g = torch.Generator().manual_seed(seed)
    shapes = {"self_attn.qkv": (3 * dim, dim), "self_attn.o": (dim, dim), "cross_attn.q": (dim, dim),
              "cross_attn.k": (dim, dim), "cross_attn.v": (dim, dim), "cross_attn.o": (dim, dim),
              "ffn.0": (ffn, dim), "ffn.2": (dim, ffn)}
    parts = {}
    for name, (N, K) in shapes.items():
        q, _, sw = ow.weight((torch.randn(N, K, generator=g) * 0.02).numpy())
        parts[name] = dict(qweight=ow.pack_nibbles(q), wscales=sw, bias=(torch.randn(N, generator=g) * 0.02).numpy())
    return parts


def test_row_subset_equals_the_whole_chunk():
    dim, heads, ffn, grid, at, text = 256, 2, 512, (3, 4, 12), 96, 40
    n = grid[0] * grid[1] * grid[2]  # 144 tokens: four whole blocks of 32 and a short one of 16
    parts = random_parts(dim, ffn, 0)
    g = torch.Generator().manual_seed(1)
    X = torch.randn(n, dim, generator=g).numpy()
    mod = (torch.randn(6, dim, generator=g) * 0.1).numpy()
    ctx = torch.randn(text, dim, generator=g).to(torch.bfloat16).float().numpy()
    cap = at + n
    ck, cks = of.quantize_rows((torch.randn(1, cap, heads, 128, generator=g) + 0.3).numpy())
    cv, cvs = of.quantize_rows(torch.randn(1, cap, heads, 128, generator=g).numpy())
    norms = dict(norm_q=np.ones(dim, np.float32) * 1.1, norm_k=np.ones(dim, np.float32) * 0.9,
                 cross_norm_q=np.ones(dim, np.float32), cross_norm_k=np.ones(dim, np.float32),
                 norm3_w=np.ones(dim, np.float32), norm3_b=np.zeros(dim, np.float32))
    freq = orope.table(1024).astype(np.float32)
    args = lambda: (X, mod, parts, norms, dict(k=ck.copy(), ks=cks.copy(), v=cv.copy(), vs=cvs.copy()), at, freq,  # noqa: E731
                    grid, at // (grid[1] * grid[2]), ctx, heads)
    full_trace, sub_trace = {}, {}
    full = ob.block(*args(), trace=full_trace)
    rows = np.r_[32:64, 128:144]
    sub = ob.block(*args(), trace=sub_trace, rows=rows)
    np.testing.assert_array_equal(sub, full[rows])
    for name in ("attn", "x_after_self", "cq", "cattn", "x_after_cross", "hcodes"):
        np.testing.assert_array_equal(sub_trace[name], full_trace[name][rows])
    np.testing.assert_array_equal(sub_trace["hscales"], full_trace["hscales"][:, rows])
    with pytest.raises(ValueError):
        ob.whole_blocks(np.r_[16:48], n)


def test_gemm_is_the_sum_of_scaled_integer_partials():
    g = torch.Generator().manual_seed(2)
    M, N, K = 40, 48, 256
    xq = torch.randint(-8, 8, (M, K), generator=g).numpy()
    wq = torch.randint(-8, 8, (N, K), generator=g).numpy()
    sx = ow.round_to(torch.rand(K // 64, M, generator=g).numpy() + 0.1, "bfloat16")
    sw = ow.round_to(torch.rand(K // 64, N, generator=g).numpy() * 0.01, "bfloat16")
    P = ow.group_partials(xq, wq).astype(np.float32)
    want = np.zeros((M, N), np.float32)
    for gi in range(K // 64):
        want += P[gi] * (sx[gi][:, None] * sw[gi][None, :]).astype(np.float32)
    np.testing.assert_array_equal(ow.gemm(xq, sx, wq, sw), want)
