"""The drop-in, end to end: the reference's own modules (the wan_dit_lab package, unmodified, installed into
baseline/_ref by baseline/install_reference.sh) run on this build's kernels once integration.install has rebound
their call sites (rope, kv_store, w4a4, attention, operators; the reference's runtime/pipeline.py:92-122 swap
points). The reference's PackedW4A4Linear (quantization/w4a4.py:220-231) over parts made by the reference's
quantize, and its FusedQKVAttention (w4a4.py:248-262) with RMSNorm, RoPE and KVCache(sage=True, fp8=True).attend
(generation/causal.py:193-220) over a cache that already holds keys, must give what this build's own functions
give on the same inputs, bit for bit: the same kernels, reached through the reference's call sites with its
argument conventions. The rebound RoPE equals the reference's own torch rope_apply, and restore() puts every
original back. Skipped where the reference package is not installed."""

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "wan_dit_lab").is_dir(),
                                 reason="the reference package is not installed (baseline/install_reference.sh)")]


@pytest.fixture(scope="module")
def ref():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from wan_dit_lab.generation import causal
    from wan_dit_lab.kernels import operators, sage_kv
    from wan_dit_lab.models import multi_head_attention, rope
    from wan_dit_lab.quantization import w4a4
    return dict(causal=causal, operators=operators, sage_kv=sage_kv, attention=multi_head_attention, rope=rope,
                w4a4=w4a4)


def seeded(shape, seed, scale=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * scale


def freq_table(rope_mod, d=128):
    """The reference's float32 RoPE table (2, position, pair): time / height / width pairs 22 / 21 / 21."""
    return torch.cat([rope_mod.rope(1024, d - 4 * (d // 6)), rope_mod.rope(1024, 2 * (d // 6)),
                      rope_mod.rope(1024, 2 * (d // 6))], dim=-1).float().cuda()


def test_install_rebinds_and_restores(ref):
    from wan_dit_lab_b200 import integration
    from wan_dit_lab_b200.kernels import rope as our_rope
    originals = (ref["attention"].rope_apply, ref["w4a4"].w4a4_linear, ref["sage_kv"].attend, ref["operators"].load,
                 ref["causal"].KVCache.store)
    restore = integration.install(integration.STEPS, attention=ref["attention"], w4a4=ref["w4a4"],
                                  causal=ref["causal"], sage_kv=ref["sage_kv"], operators=ref["operators"])
    try:
        assert ref["attention"].rope_apply is our_rope.rope_apply and ref["w4a4"].rope_apply is our_rope.rope_apply
        assert ref["sage_kv"].attend is not originals[2] and ref["operators"].load is not originals[3]
        # the rebound RoPE against the reference's own torch rope_apply on the same chunk
        x = seeded((1, 2 * 4 * 8, 4, 128), 1).cuda()
        freq = freq_table(ref["rope"])
        got = ref["attention"].rope_apply(x, [(2, 4, 8)], freq, 3)
        want = originals[0](x, [(2, 4, 8)], freq, 3)
        assert torch.allclose(got, want, rtol=0, atol=1e-5), float((got - want).abs().max())
    finally:
        restore()
    now = (ref["attention"].rope_apply, ref["w4a4"].w4a4_linear, ref["sage_kv"].attend, ref["operators"].load,
           ref["causal"].KVCache.store)
    assert all(a is b for a, b in zip(now, originals))


@pytest.fixture
def installed(ref):
    from wan_dit_lab_b200 import integration
    restore = integration.install(integration.STEPS, attention=ref["attention"], w4a4=ref["w4a4"],
                                  causal=ref["causal"], sage_kv=ref["sage_kv"], operators=ref["operators"])
    yield ref
    restore()


@pytest.mark.parametrize("rank", [0, 32])
def test_reference_packed_linear_runs_on_the_b200_kernels(installed, rank):
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.quantization import w4a4
    rw = installed["w4a4"]
    N, K = 768, 1024
    W, b = seeded((N, K), 2, 0.02).cuda(), seeded((N,), 3, 0.1).cuda()
    parts = rw.quantize(W, b, rank=rank)  # the reference's name, this build's quantize
    layer = rw.PackedW4A4Linear(**parts)
    X = seeded((2, 150, K), 4).to(torch.bfloat16).cuda()
    got = layer(X)
    want = w4a4.linear(X.reshape(-1, K), parts).reshape(2, 150, N)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert got.shape == (2, 150, N) and torch.equal(got, want)


def test_reference_attention_block_over_its_kv_cache(installed):
    """The reference's FusedQKVAttention with its KVCache(sage=True, fp8=True), the cache holding `at` keys of
    earlier frames: one chunk's self-attention through the reference's modules, against the same steps taken
    with this build's functions."""
    from wan_dit_lab_b200 import _native
    from wan_dit_lab_b200.kernels import cache_fp8, rope as our_rope, sage_kv
    from wan_dit_lab_b200.quantization import w4a4
    rw, rc = installed["w4a4"], installed["causal"]
    dim, heads, frames, h, w = 1024, 8, 2, 4, 8
    n, at, start = frames * h * w, 128, 2
    att = rw.FusedQKVAttention(dim, heads)
    with torch.no_grad():
        att.norm_q.weight.copy_(1 + seeded((dim,), 5, 0.1))
        att.norm_k.weight.copy_(1 + seeded((dim,), 6, 0.1))
    qkv = rw.quantize(seeded((3 * dim, dim), 7, 0.02).cuda(), seeded((3 * dim,), 8, 0.1).cuda(), rank=0)
    o = rw.quantize(seeded((dim, dim), 9, 0.02).cuda(), seeded((dim,), 10, 0.1).cuda(), rank=0)
    att.qkv, att.o = rw.PackedW4A4Linear(**qkv), rw.PackedW4A4Linear(**o)
    att = att.cuda()
    freq = freq_table(installed["rope"])
    X = seeded((1, n, dim), 11).cuda()
    Kc = (seeded((1, at, heads, 128), 12) + 0.3).cuda()  # keys and values of the earlier frames
    Vc = seeded((1, at, heads, 128), 13).cuda()

    cache = rc.KVCache(at + 2 * n, sage=True, fp8=True, chunk=frames)
    cache.allocate(Vc[:, :n])
    cache.store(0, Kc, Vc)  # the rebound store: this build's FP8 store
    cache.saved = at
    with torch.no_grad():
        got = att(X, grid_sizes=[(frames, h, w)], freq=freq, start_frame=start, cache=cache)

    # the same steps with this build's functions, over a cache of its own
    with torch.no_grad():
        q, k, v = w4a4.linear(X.reshape(n, dim).to(torch.bfloat16), qkv).reshape(1, n, 3 * dim).split(dim, dim=-1)
        Q = our_rope.rope_apply(att.norm_q(q).reshape(1, n, heads, 128), [(frames, h, w)], freq, start)
        K = our_rope.rope_apply(att.norm_k(k).reshape(1, n, heads, 128), [(frames, h, w)], freq, start)
        V = v.reshape(1, n, heads, 128)
        cap = at + 3 * n
        ck = torch.empty(1, cap, heads, 128, dtype=torch.float8_e4m3fn, device="cuda")
        cv = torch.empty_like(ck)
        cks = torch.empty(1, cap, heads, 1, device="cuda")
        cvs = torch.empty_like(cks)
        cache_fp8.store_kv_fp8(Kc, Vc, ck, cks, cv, cvs, 0)
        cache_fp8.store_kv_fp8(K, V, ck, cks, cv, cvs, at)
        A = sage_kv.attend(Q, ck, cks, cv, cvs, at, K, V)
        want = w4a4.linear(A.reshape(n, dim), o).reshape(1, n, dim)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert got.shape == want.shape and torch.equal(got, want)
    # the reference's cache holds the chunk where this build's store put it
    assert torch.equal(cache.k[:, at:at + n].view(torch.uint8), ck[:, at:at + n].view(torch.uint8))
