"""The tensor-parallel block (models/block_tp.py) against the whole block on one GPU: its shards run in one process
in lock step (run_lockstep sums what they yield, as the NCCL all-reduce does across GPUs), on the same packed
weights, inputs, prompt and FP8 cache. The shards' residual streams are equal to each other bit for bit and to
the whole block's within relative L2 1e-2 of the block's update (float32 sums in another order: the row-parallel
partial products, the low-rank branches' shares and the RMS statistics, whose rare bf16 rounding differences the
INT4 requantizations downstream turn into code steps), their cache rows equal the whole cache's heads in >= 99.9 % of bytes.
Also the kernels the split adds: fp32 partial GEMMs (their sum is the whole product; partial + wdl_residual_update
equals the residual epilogue bit for bit), column counts that are multiples of 128 in the folded GEMM, sharded RMS
statistics."""

import numpy as np
import pytest
import torch

from oracle import fp8 as of
from oracle import rope as orope

pytestmark = pytest.mark.gpu


def native():
    from wan_dit_lab_b200 import _native
    return _native


def random_state(dim, ffn, seed):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02  # noqa: E731
    st = {}
    for attn in ("self_attn", "cross_attn"):
        for name in ("q", "k", "v", "o"):
            st[f"{attn}.{name}.weight"], st[f"{attn}.{name}.bias"] = r(dim, dim), r(dim)
        st[f"{attn}.norm_q.weight"] = 1 + r(dim) * 5
        st[f"{attn}.norm_k.weight"] = 1 + r(dim) * 5
    st["ffn.0.weight"], st["ffn.0.bias"] = r(ffn, dim), r(ffn)
    st["ffn.2.weight"], st["ffn.2.bias"] = r(dim, ffn), r(dim)
    st["norm3.weight"], st["norm3.bias"] = 1 + r(dim) * 5, r(dim)
    st["modulation"] = torch.randn(1, 6, dim, generator=g) / dim ** 0.5
    return st


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("dim,heads,ffn,world,frames,h,w,at,text,rank", [
    (1024, 8, 4096, 2, 2, 4, 8, 128, 32, 0),
    (1024, 8, 4096, 4, 2, 4, 8, 128, 32, 0),
    (3072, 24, 14336, 8, 2, 4, 16, 256, 64, 0),
    (1024, 8, 4096, 2, 2, 4, 8, 128, 32, 32),
    (1024, 8, 4096, 4, 2, 4, 8, 128, 32, 32),
])
def test_tp_block_matches_whole_block(dim, heads, ffn, world, frames, h, w, at, text, rank):
    """rank 32: SVDQuant low-rank branches and smoothing on every layer; the row shards' shares of each branch
    are summed with their partial products."""
    import sys
    from pathlib import Path
    from wan_dit_lab_b200.models.block import WanBlockB200, quantize_block
    from wan_dit_lab_b200.models.block_tp import WanBlockTP, run_lockstep
    _native = native()
    n = frames * h * w
    state = random_state(dim, ffn, 11)
    if rank:
        sys.path.insert(0, str(Path(__file__).resolve().parent))
        from test_block_gpu import lowrank_parts
        parts = lowrank_parts(state, rank, 13)
    else:
        parts = quantize_block({k: v.cuda() for k, v in state.items()})
    whole = WanBlockB200(state, dim, ffn, heads, parts=parts)
    shards = [WanBlockTP(state, dim, ffn, heads, r, world, parts=parts) for r in range(world)]
    assert all(s.code_format == whole.code_format and s.lowrank == bool(rank) for s in shards)
    g = torch.Generator().manual_seed(12)
    X = torch.randn(n, dim, generator=g).cuda()
    time_in = (torch.randn(6, dim, generator=g) * 0.1).cuda()
    ctx = torch.randn(text, dim, generator=g).to(torch.bfloat16).cuda()
    cap = at + n + 16
    ck8, cks = of.quantize_rows((torch.randn(1, cap, heads, 128, generator=g) + 0.3).numpy())
    cv8, cvs = of.quantize_rows(torch.randn(1, cap, heads, 128, generator=g).numpy())
    cache = [torch.from_numpy(a).cuda() for a in (ck8[0], cks[0, ..., 0], cv8[0], cvs[0, ..., 0])]
    freq = torch.from_numpy(orope.table(1024).astype(np.float32)).cuda()
    grid, start = (frames, h, w), at // (h * w)

    Xw = X.clone()
    whole_cache = [t.clone() for t in cache]
    buf = whole.buffers(n, at + n, text, "cuda")
    whole.forward(Xw, whole.modulation_of(time_in), (*whole_cache, cap), at, freq, grid, start, whole.cross_kv(ctx),
                  buf)

    hl = heads // world
    xs, caches, gens = [], [], []
    for r, blk in enumerate(shards):
        c = [t[:, r * hl:(r + 1) * hl].contiguous() for t in cache]
        xr = X.clone()
        xs.append(xr)
        caches.append(c)
        gens.append(blk.steps(xr, blk.modulation_of(time_in), (*c, cap), at, freq, grid, start, blk.cross_kv(ctx),
                              blk.buffers(n, at + n, text, "cuda")))
    run_lockstep(gens)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    for xr in xs[1:]:
        assert torch.equal(xr, xs[0])
    err = rel((xs[0] - X).cpu().numpy(), (Xw - X).cpu().numpy())
    print(f"world {world}, rank {rank}: block update vs whole block, relative L2 {err:.2e}")
    # The row-parallel partial products are summed in another order than the whole GEMM's accumulation, so a few
    # bf16 roundings of O's output come out the other way (the stream after self-attention: ~3e-5 apart); the INT4
    # requantizations downstream (the FFN input, its unsigned hidden codes) turn such rows' small differences into
    # whole code steps (measured at 8 shards of config 3: hidden codes 99.98 % equal, the update 1.7e-3 apart).
    # The shards are held to the stage bar of a linear layer, 1e-2.
    assert err <= 1e-2
    for r, c in enumerate(caches):
        for i in (0, 2):
            got = c[i][at:at + n].cpu()
            ref = whole_cache[i][at:at + n, r * hl:(r + 1) * hl].cpu()
            assert (got == ref).float().mean() >= 0.999


@pytest.mark.parametrize("world", [2, 4])
def test_tp_block_with_forcing_kv_split_matches_whole_block(world):
    """Forcing-KV's head split on shards: each shard attends with the static heads among its own (renumbered),
    the others to the whole window; the result equals the whole block's with the same split within relative L2
    1e-3 of the update, and the shards' residual streams are equal bit for bit."""
    from wan_dit_lab_b200.models.block import WanBlockB200, quantize_block
    from wan_dit_lab_b200.models.block_tp import WanBlockTP, run_lockstep
    _native = native()
    dim, heads, ffn, frames, h, w, at, text = 1024, 8, 4096, 2, 4, 8, 192, 32
    n = frames * h * w
    state = random_state(dim, ffn, 15)
    parts = quantize_block({k: v.cuda() for k, v in state.items()})
    g = torch.Generator().manual_seed(16)
    X = torch.randn(n, dim, generator=g).cuda()
    time_in = (torch.randn(6, dim, generator=g) * 0.1).cuda()
    ctx = torch.randn(text, dim, generator=g).to(torch.bfloat16).cuda()
    cap = at + n
    ck8, cks = of.quantize_rows((torch.randn(1, cap, heads, 128, generator=g) + 0.3).numpy())
    cv8, cvs = of.quantize_rows(torch.randn(1, cap, heads, 128, generator=g).numpy())
    cache = [torch.from_numpy(a).cuda() for a in (ck8[0], cks[0, ..., 0], cv8[0], cvs[0, ..., 0])]
    freq = torch.from_numpy(orope.table(1024).astype(np.float32)).cuda()
    grid, start = (frames, h, w), at // (h * w)
    anchors = torch.cat([torch.arange(32), torch.arange(at - 32, at)]).to(torch.int32).cuda()  # a sink, a frame
    static = [1, 5, 6]

    def split(heads_here, first):
        st = [x - first for x in static if first <= x < first + heads_here]
        dy = [x for x in range(heads_here) if x not in st]
        as_int = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
        return as_int(st), as_int(dy), anchors

    whole = WanBlockB200(state, dim, ffn, heads, parts=parts)
    Xw = X.clone()
    whole.forward(Xw, whole.modulation_of(time_in), (*[t.clone() for t in cache], cap), at, freq, grid, start,
                  whole.cross_kv(ctx), whole.buffers(n, cap, text, "cuda"), forcing=split(heads, 0))
    plain = X.clone()
    whole.forward(plain, whole.modulation_of(time_in), (*[t.clone() for t in cache], cap), at, freq, grid, start,
                  whole.cross_kv(ctx), whole.buffers(n, cap, text, "cuda"))
    hl = heads // world
    xs, gens = [], []
    for r in range(world):
        blk = WanBlockTP(state, dim, ffn, heads, r, world, parts=parts)
        c = [t[:, r * hl:(r + 1) * hl].contiguous() for t in cache]
        xr = X.clone()
        xs.append(xr)
        gens.append(blk.steps(xr, blk.modulation_of(time_in), (*c, cap), at, freq, grid, start, blk.cross_kv(ctx),
                              blk.buffers(n, cap, text, "cuda"), forcing=split(hl, r * hl)))
    run_lockstep(gens)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    for xr in xs[1:]:
        assert torch.equal(xr, xs[0])
    d_tp, d_whole = (xs[0] - X).cpu().numpy(), (Xw - X).cpu().numpy()
    assert rel(d_tp, d_whole) <= 1e-3
    assert rel((plain - X).cpu().numpy(), d_whole) > 2e-3  # the split changed the block's output


def quantized_operands(M, N, K, seed, fmt):
    """Activation codes / scales in the GEMM's format (through the quantizer) and a prepared layer."""
    from wan_dit_lab_b200.quantization import w4a4
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=g)).to(torch.bfloat16).cuda()
    W = torch.randn(N, K, generator=g) * 0.02
    b = torch.randn(N, generator=g) * 0.1
    parts = w4a4.quantize(W.cuda(), b.cuda(), rank=0)
    layer = w4a4.PreparedW4A4(*(parts[p] for p in w4a4.PARTS), code_format=fmt)
    work = torch.empty(native().lib().wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device="cuda")
    codes, scales = layer.quantize_input(x, work)
    return x, parts, layer, codes, scales


@pytest.mark.parametrize("fmt", ["f16fold", "e4m3"])
def test_partial_gemms_sum_to_whole_and_residual_update_matches_epilogue(fmt):
    from wan_dit_lab_b200.models.block_tp import shard_rows
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    lib, st = _native.lib(), _native.stream()
    M, N, K, world = 300, 768, 2048, 4
    x, parts, layer, codes, scales = quantized_operands(M, N, K, 21, fmt)
    fc = layer.code_format
    whole = torch.empty(M, N, device="cuda")
    _native.check(lib.wdl_w4a4_gemm_f32(codes.data_ptr(), scales.data_ptr(), layer.codes.data_ptr(),
                                        layer.scales.data_ptr(), fc, None, None, 0, M, N, K, whole.data_ptr(), N, st))
    total = torch.zeros(M, N, device="cuda")
    work = torch.empty(lib.wdl_w4a4_linear_workspace(M, K), dtype=torch.uint8, device="cuda")
    for r in range(world):
        k0, k1 = r * K // world, (r + 1) * K // world
        sp, bias = shard_rows(parts, k0, k1)
        sl = w4a4.PreparedW4A4(*(sp[p] for p in w4a4.PARTS), code_format=fmt)
        c, s = sl.quantize_input(x[:, k0:k1].contiguous(), work)
        part = torch.empty(M, N, device="cuda")
        _native.check(lib.wdl_w4a4_gemm_f32(c.data_ptr(), s.data_ptr(), sl.codes.data_ptr(), sl.scales.data_ptr(),
                                            sl.code_format, None, None, 0, M, N, k1 - k0, part.data_ptr(), N, st))
        total += part
    assert rel(total.cpu().numpy(), whole.cpu().numpy()) <= 1e-6
    # partial + residual update == the GEMM's residual epilogue, bit for bit
    g = torch.Generator().manual_seed(22)
    resid = torch.randn(M, N, generator=g).cuda()
    gate = torch.randn(N, generator=g).cuda()
    want = torch.empty(M, N, device="cuda")
    _native.check(lib.wdl_w4a4_gemm_residual(codes.data_ptr(), scales.data_ptr(), layer.codes.data_ptr(),
                                             layer.scales.data_ptr(), fc, layer.bias.data_ptr(), gate.data_ptr(),
                                             resid.data_ptr(), N, M, N, K, want.data_ptr(), N, st))
    got = resid.clone()
    _native.check(lib.wdl_residual_update(whole.data_ptr(), N, layer.bias.data_ptr(), gate.data_ptr(), got.data_ptr(),
                                          N, M, N, st))
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert _native.device_error() == 0


@pytest.mark.parametrize("N", [384, 640, 1152])
def test_fold_gemm_column_counts_multiple_of_128(N):
    """N % 256 == 128: the last column tile's second half is absent (zero-filled weights, no stores)."""
    from wan_dit_lab_b200.quantization import w4a4
    _native = native()
    lib, st = _native.lib(), _native.stream()
    M, K = 200, 512
    Np = N + 128
    x, parts, big, codes, scales = quantized_operands(M, Np, K, 31, "f16fold")
    assert big.code_format == _native.CODES_F16_FOLD
    sub = {p: v for p, v in parts.items()}
    sub["qweight"], sub["wscales"], sub["bias"] = parts["qweight"][:N], parts["wscales"][:, :N], parts["bias"][:N]
    small = w4a4.PreparedW4A4(*(sub[p] for p in w4a4.PARTS), code_format="f16fold")
    small.codes, small.scales = big.codes[:N].contiguous(), big.scales  # the same folded weights and 2^F
    y_big = torch.empty(M, Np, dtype=torch.bfloat16, device="cuda")
    _native.check(lib.wdl_w4a4_gemm(codes.data_ptr(), scales.data_ptr(), big.codes.data_ptr(), big.scales.data_ptr(),
                                    big.code_format, big.bias.data_ptr(), M, Np, K, y_big.data_ptr(), Np, st))
    y = torch.full((M, Np), 7.0, dtype=torch.bfloat16, device="cuda")  # columns N.. must stay untouched
    _native.check(lib.wdl_w4a4_gemm(codes.data_ptr(), scales.data_ptr(), small.codes.data_ptr(),
                                    small.scales.data_ptr(), small.code_format, small.bias.data_ptr(), M, N, K,
                                    y.data_ptr(), Np, st))
    torch.cuda.synchronize()
    assert torch.equal(y[:, :N], y_big[:, :N])
    assert bool((y[:, N:] == 7.0).all())
    assert _native.device_error() == 0


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_rms_statistics(world):
    """wdl_rows_sumsq over each shard's heads, summed, drives wdl_qkv_prep_sharded / wdl_rms_rows_sharded to the
    whole row's normalization: q / k / cache rows and the cross query equal the whole-row kernels' in >= 99.9 %."""
    _native = native()
    lib, st = _native.lib(), _native.stream()
    heads, n, h, w = 6, 64, 4, 8
    dim, d = heads * 128, heads * 128 // world
    g = torch.Generator().manual_seed(41)
    qkv = torch.randn(n, 3 * dim, generator=g).to(torch.bfloat16).cuda()
    nq = (1 + torch.randn(dim, generator=g) * 0.1).cuda()
    nk = (1 + torch.randn(dim, generator=g) * 0.1).cuda()
    freq = torch.from_numpy(orope.table(64).astype(np.float32)).cuda()
    cap = n
    q = torch.empty(n, dim, device="cuda")
    k = torch.empty(n, dim, device="cuda")
    ck = torch.zeros(cap, heads, 128, dtype=torch.uint8, device="cuda")
    cks = torch.zeros(cap, heads, device="cuda")
    cv, cvs = torch.zeros_like(ck), torch.zeros_like(cks)
    _native.check(lib.wdl_qkv_prep_sharded(qkv.data_ptr(), 3 * dim, n, dim, nq.data_ptr(), nk.data_ptr(), 1e-6, None,
                                           dim, freq.data_ptr(), 64, h, w, 0, q.data_ptr(), k.data_ptr(),
                                           ck.data_ptr(), cks.data_ptr(), cv.data_ptr(), cvs.data_ptr(), cap, 0, st))
    hl = heads // world
    shards = []
    total = torch.zeros(n, 2, device="cuda")
    for r in range(world):
        cols = torch.cat([torch.arange(r * d, (r + 1) * d) + j * dim for j in range(3)]).cuda()
        part = qkv.index_select(1, cols).contiguous()
        s = torch.empty(n, 2, device="cuda")
        _native.check(lib.wdl_rows_sumsq(part.data_ptr(), 3 * d, n, d, 2, d, s.data_ptr(), st))
        total += s
        shards.append(part)
    ok = []
    for r, part in enumerate(shards):
        qs, ks = torch.empty(n, d, device="cuda"), torch.empty(n, d, device="cuda")
        c = [torch.zeros(cap, hl, 128, dtype=torch.uint8, device="cuda"), torch.zeros(cap, hl, device="cuda")]
        c += [torch.zeros_like(c[0]), torch.zeros_like(c[1])]
        sl = slice(r * d, (r + 1) * d)
        _native.check(lib.wdl_qkv_prep_sharded(part.data_ptr(), 3 * d, n, d, nq[sl].contiguous().data_ptr(),
                                               nk[sl].contiguous().data_ptr(), 1e-6, total.data_ptr(), dim,
                                               freq.data_ptr(), 64, h, w, 0, qs.data_ptr(), ks.data_ptr(),
                                               c[0].data_ptr(), c[1].data_ptr(), c[2].data_ptr(), c[3].data_ptr(),
                                               cap, 0, st))
        torch.cuda.synchronize()
        ok += [(qs == q[:, sl]).float().mean().item(), (ks == k[:, sl]).float().mean().item(),
               (c[0] == ck[:, r * hl:(r + 1) * hl]).float().mean().item(),
               (c[2] == cv[:, r * hl:(r + 1) * hl]).float().mean().item()]
    assert min(ok) >= 0.999, ok
    # the cross query's RMSNorm over shards
    x = torch.randn(n, dim, generator=g).to(torch.bfloat16).cuda()
    wq = (1 + torch.randn(dim, generator=g) * 0.1).cuda()
    full = torch.empty(n, dim, device="cuda")
    _native.check(lib.wdl_rms_rows_sharded(x.data_ptr(), dim, n, dim, wq.data_ptr(), 1e-6, None, dim, full.data_ptr(),
                                           dim, st))
    ss = torch.zeros(n, device="cuda")
    for r in range(world):
        s = torch.empty(n, device="cuda")
        _native.check(lib.wdl_rows_sumsq(x[:, r * d:].data_ptr(), dim, n, d, 1, 0, s.data_ptr(), st))
        ss += s
    for r in range(world):
        out = torch.empty(n, d, device="cuda")
        _native.check(lib.wdl_rms_rows_sharded(x[:, r * d:].data_ptr(), dim, n, d, wq[r * d:].data_ptr(), 1e-6,
                                               ss.data_ptr(), dim, out.data_ptr(), d, st))
        torch.cuda.synchronize()
        assert (out == full[:, r * d:(r + 1) * d]).float().mean().item() >= 0.999
    expected = x.float() * torch.rsqrt(x.float().pow(2).mean(1, keepdim=True) + 1e-6)
    assert rel((full / wq).cpu().numpy(), expected.to(torch.bfloat16).float().cpu().numpy()) <= 1e-2
    assert _native.device_error() == 0
