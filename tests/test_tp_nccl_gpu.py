"""The tensor-parallel block across GPUs: one process per GPU, NCCL all-reduce as the reduce callable
(WanBlockTP.forward). Every rank ends with the same residual stream, equal bit for bit to what the shards give in
lock step on one GPU (the same sums: NCCL adds two ranks' values in one order) and within relative L2 1e-3 of the
whole block's update; the same forward captured in a CUDA graph (its all-reduces with it, as the rollout's passes
are) and replayed gives the eager result bit for bit. Needs two GPUs; skipped otherwise."""

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(dim, heads, ffn, frames, h, w, at, text):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle import fp8 as of
    from oracle import rope as orope
    from test_block_tp_gpu import random_state
    n = frames * h * w
    state = random_state(dim, ffn, 51)
    g = torch.Generator().manual_seed(52)
    X = torch.randn(n, dim, generator=g)
    time_in = torch.randn(6, dim, generator=g) * 0.1
    ctx = torch.randn(text, dim, generator=g).to(torch.bfloat16)
    cap = at + n + 16
    ck8, cks = of.quantize_rows((torch.randn(1, cap, heads, 128, generator=g) + 0.3).numpy())
    cv8, cvs = of.quantize_rows(torch.randn(1, cap, heads, 128, generator=g).numpy())
    cache = [torch.from_numpy(a) for a in (ck8[0], cks[0, ..., 0], cv8[0], cvs[0, ..., 0])]
    freq = torch.from_numpy(orope.table(1024).astype(np.float32))
    return state, X, time_in, ctx, cache, cap, freq, n


CASE = (1024, 8, 4096, 2, 4, 8, 128, 32)


def _rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT / "wan-dit-lab_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from wan_dit_lab_b200 import _native
        from wan_dit_lab_b200.models.block import quantize_block
        from wan_dit_lab_b200.models.block_tp import WanBlockTP
        dim, heads, ffn, frames, h, w, at, text = CASE
        state, X, time_in, ctx, cache, cap, freq, n = _setup(*CASE)
        parts = quantize_block({k: v.to(dev) for k, v in state.items()})
        blk = WanBlockTP(state, dim, ffn, heads, rank, world, device=dev, parts=parts,
                         reduce=lambda t: dist.all_reduce(t))
        hl = heads // world
        c = [t[:, rank * hl:(rank + 1) * hl].contiguous().to(dev) for t in cache]
        Xd = X.to(dev)
        args = (blk.modulation_of(time_in.to(dev)), (*c, cap), at, freq.to(dev), (frames, h, w), at // (h * w),
                blk.cross_kv(ctx.to(dev)), blk.buffers(n, at + n, text, dev))
        blk.forward(Xd, *args)
        torch.cuda.synchronize()
        # the same pass captured with its all-reduces (every rank captures and replays the same collectives in the
        # same order) and replayed from the same input: it writes the same cache rows with the same values
        Xg = X.to(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            blk.forward(Xg, *args)
        Xg.copy_(X.to(dev))
        graph.replay()
        torch.cuda.synchronize()
        replay_equal = bool(torch.equal(Xg, Xd))
        del graph  # released before the process group (it holds NCCL calls)
        torch.cuda.synchronize()
        out[rank] = (Xd.cpu().numpy(), _native.device_error(), replay_equal)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_block_over_nccl_matches_lockstep_and_whole_block():
    from wan_dit_lab_b200.models.block import Buffers, WanBlockB200, quantize_block
    from wan_dit_lab_b200.models.block_tp import WanBlockTP, run_lockstep
    world, port = 2, free_port()
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
    x0, err0, replay0 = out[0]
    x1, err1, replay1 = out[1]
    assert err0 == 0 and err1 == 0
    assert replay0 and replay1  # graph replay with the all-reduces captured equals the eager pass
    np.testing.assert_array_equal(x0, x1)
    # the same split in lock step on this GPU, and the whole block
    dim, heads, ffn, frames, h, w, at, text = CASE
    state, X, time_in, ctx, cache, cap, freq, n = _setup(*CASE)
    parts = quantize_block({k: v.cuda() for k, v in state.items()})
    freq = freq.cuda()
    hl = heads // world
    xs, gens = [], []
    for r in range(world):
        blk = WanBlockTP(state, dim, ffn, heads, r, world, parts=parts)
        c = [t[:, r * hl:(r + 1) * hl].contiguous().cuda() for t in cache]
        xr = X.cuda()
        xs.append(xr)
        gens.append(blk.steps(xr, blk.modulation_of(time_in.cuda()), (*c, cap), at, freq, (frames, h, w),
                              at // (h * w), blk.cross_kv(ctx.cuda()), blk.buffers(n, at + n, text, "cuda")))
    run_lockstep(gens)
    np.testing.assert_array_equal(xs[0].cpu().numpy(), x0)
    whole = WanBlockB200(state, dim, ffn, heads, parts=parts)
    Xw = X.cuda()
    whole.forward(Xw, whole.modulation_of(time_in.cuda()), (*[t.cuda() for t in cache], cap), at, freq,
                  (frames, h, w), at // (h * w), whole.cross_kv(ctx.cuda()), Buffers(n, dim, ffn, heads, at + n, text,
                                                                                       "cuda"))
    d_tp, d_whole = x0 - X.numpy(), (Xw.cpu() - X).numpy()
    assert np.linalg.norm(d_tp - d_whole) / np.linalg.norm(d_whole) <= 1e-3
