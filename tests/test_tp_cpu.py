"""The tensor-parallel split's host logic on CPU (models/block_tp.py): sharding the packed W4A4 parts of a block,
checked with the oracle (column shards give the whole layer's columns bit for bit, row shards' partial products
sum to the whole product and keep the bias aside), the lock-step driver, and the all-reduce of the shards'
partials across two gloo ranks (each rank one shard, as the NCCL ranks are on GPUs)."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4a4 as ow

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "wan-dit-lab_b200"))


def packed(W, bias, seed):
    """A layer's parts in the package's logical packed format, built with the oracle on the CPU."""
    codes, _, scales = ow.weight(W)
    N, K = W.shape
    return dict(qweight=torch.from_numpy(ow.pack_nibbles(codes)), wscales=torch.from_numpy(scales).to(torch.bfloat16),
                proj_down=torch.zeros(K, 0, dtype=torch.bfloat16), proj_up=torch.zeros(N, 0, dtype=torch.bfloat16),
                smooth=None, bias=torch.from_numpy(bias).to(torch.bfloat16))


def block_parts(dim, ffn, seed):
    rng = np.random.default_rng(seed)
    w = lambda n, k: (rng.standard_normal((n, k)) * 0.02).astype(np.float32)  # noqa: E731
    b = lambda n: (rng.standard_normal(n) * 0.1).astype(np.float32)  # noqa: E731
    shapes = {"self_attn.qkv": (3 * dim, dim), "self_attn.o": (dim, dim), "cross_attn.q": (dim, dim),
              "cross_attn.k": (dim, dim), "cross_attn.v": (dim, dim), "cross_attn.o": (dim, dim),
              "ffn.0": (ffn, dim), "ffn.2": (dim, ffn)}
    return {name: packed(w(n, k), b(n), seed) for name, (n, k) in shapes.items()}


def oracle_product(parts, x):
    """The oracle's W4A4 product of x [M, K] (bf16 values) by a layer's parts, without bias, float32."""
    codes = ow.unpack_nibbles(parts["qweight"].numpy())
    _, xq, sx = ow.linear(x, codes, parts["wscales"].float().numpy())
    return ow.gemm(xq, sx, codes, parts["wscales"].float().numpy())


def test_shards_partition_every_layer():
    from wan_dit_lab_b200.models.block_tp import ROW_PARALLEL, shard_block_parts
    dim, heads, ffn, world, M = 256, 2, 512, 2, 20
    parts = block_parts(dim, ffn, 1)
    x = ow.round_to(np.random.default_rng(2).standard_normal((M, dim)).astype(np.float32), "bfloat16")
    h = ow.round_to(np.random.default_rng(3).standard_normal((M, ffn)).astype(np.float32), "bfloat16")
    whole = {name: oracle_product(parts[name], h if name == "ffn.2" else x) for name in parts}
    shards = [shard_block_parts(parts, dim, ffn, heads, r, world) for r in range(world)]
    d, f = dim // world, ffn // world
    for r, (sp, bias) in enumerate(shards):
        # column-parallel: this shard's heads of q, k and v (qkv), heads (cross q), hidden channels (ffn.0)
        y = oracle_product(sp["self_attn.qkv"], x)
        for j in range(3):
            np.testing.assert_array_equal(y[:, j * d:(j + 1) * d], whole["self_attn.qkv"][:, j * dim + r * d:j * dim + (r + 1) * d])
        np.testing.assert_array_equal(oracle_product(sp["cross_attn.q"], x), whole["cross_attn.q"][:, r * d:(r + 1) * d])
        np.testing.assert_array_equal(oracle_product(sp["ffn.0"], x), whole["ffn.0"][:, r * f:(r + 1) * f])
        torch.testing.assert_close(sp["ffn.0"]["bias"], parts["ffn.0"]["bias"][r * f:(r + 1) * f], rtol=0, atol=0)
        for name in ("cross_attn.k", "cross_attn.v"):
            assert sp[name] is parts[name]
        for name in ROW_PARALLEL:
            assert sp[name]["bias"] is None and bias[name] is parts[name]["bias"]
    # row-parallel: the shards' partial products (their slices of K) sum to the whole product
    for name in ROW_PARALLEL:
        inp = h if name == "ffn.2" else x
        k = inp.shape[1] // world
        total = sum(oracle_product(shards[r][0][name], inp[:, r * k:(r + 1) * k]) for r in range(world))
        rel = np.linalg.norm(total - whole[name]) / np.linalg.norm(whole[name])
        assert rel <= 1e-6, (name, rel)


def lowrank_packed(N, K, rank, seed):
    """A layer's parts with a rank-`rank` low-rank branch and a smoothing vector (random factors: the split is
    checked, not the decomposition)."""
    rng = np.random.default_rng(seed)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    parts = packed((rng.standard_normal((N, K)) * 0.02).astype(np.float32),
                   (rng.standard_normal(N) * 0.1).astype(np.float32), seed)
    parts["proj_down"] = bf(rng.standard_normal((K, rank)) * 0.05)
    parts["proj_up"] = bf(rng.standard_normal((N, rank)) * 0.05)
    parts["smooth"] = bf(rng.uniform(0.5, 2.5, K))
    return parts


def oracle_lowrank_product(parts, x):
    """The oracle's product of x by a layer with its branch and smoothing, without bias, float32."""
    f = lambda t: t.float().numpy()  # noqa: E731
    return ow.linear_lowrank(x, ow.unpack_nibbles(parts["qweight"].numpy()), f(parts["wscales"]), f(parts["proj_down"]),
                             f(parts["proj_up"]), None, f(parts["smooth"]))


def test_lowrank_branches_shard_with_their_layers():
    """Column shards keep proj_down whole and their rows of proj_up: their outputs are the whole layer's columns.
    Row shards keep their rows of proj_down and smooth: their products, branch shares included, sum to the whole
    layer's (bias kept aside, added once)."""
    from wan_dit_lab_b200.models.block_tp import shard_columns, shard_rows
    M, N, K, world, rank = 24, 256, 512, 4, 16
    x = ow.round_to(np.random.default_rng(5).standard_normal((M, K)).astype(np.float32), "bfloat16")
    parts = lowrank_packed(N, K, rank, 6)
    whole = oracle_lowrank_product(parts, x)
    n = N // world
    for r in range(world):
        sp = shard_columns(parts, torch.arange(r * n, (r + 1) * n))
        assert sp["proj_down"] is parts["proj_down"] and sp["smooth"] is parts["smooth"]
        got = oracle_lowrank_product(sp, x)
        np.testing.assert_allclose(got, whole[:, r * n:(r + 1) * n], rtol=1e-6, atol=1e-6)
    k = K // world
    total = np.zeros_like(whole)
    for r in range(world):
        sp, bias = shard_rows(parts, r * k, (r + 1) * k)
        assert bias is parts["bias"] and sp["proj_up"] is parts["proj_up"]
        assert sp["proj_down"].shape == (k, rank) and sp["smooth"].shape == (k,)
        total += oracle_lowrank_product(sp, x[:, r * k:(r + 1) * k])
    assert np.linalg.norm(total - whole) / np.linalg.norm(whole) <= 1e-6


def test_shards_reject_splits_off_group_boundaries():
    from wan_dit_lab_b200.models.block_tp import shard_block_parts, shard_rows
    parts = block_parts(256, 512, 4)
    try:
        shard_rows(parts["self_attn.o"], 0, 96)
    except ValueError:
        pass
    else:
        raise AssertionError("a row shard off a 64-channel boundary must be refused")
    try:
        shard_block_parts(parts, 256, 512, 2, 0, 3)
    except ValueError:
        pass
    else:
        raise AssertionError("3 shards of 2 heads must be refused")


def test_lockstep_replaces_each_yield_by_the_sum():
    from wan_dit_lab_b200.models.block_tp import run_lockstep
    seen = []

    def shard(r):
        a = torch.full((3,), float(r + 1))
        yield a
        seen.append(a.clone())
        b = torch.full((2, 2), 10.0 * (r + 1))
        yield b
        seen.append(b.clone())

    run_lockstep([shard(r) for r in range(3)])
    assert all(torch.equal(t, torch.full((3,), 6.0)) for t in seen[:3])
    assert all(torch.equal(t, torch.full((2, 2), 60.0)) for t in seen[3:])

    def short():
        yield torch.zeros(1)

    def long():
        yield torch.zeros(1)
        yield torch.zeros(1)

    try:
        run_lockstep([short(), long()])
    except RuntimeError:
        pass
    else:
        raise AssertionError("shards yielding different numbers of tensors must be refused")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "wan-dit-lab_b200"))
    from wan_dit_lab_b200.models.block_tp import ROW_PARALLEL, shard_block_parts
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dim, heads, ffn, M = 256, 4, 512, 12
        parts = block_parts(dim, ffn, 5)  # every rank builds the same weights from the seed
        sp, bias = shard_block_parts(parts, dim, ffn, heads, rank, world)
        x = ow.round_to(np.random.default_rng(6).standard_normal((M, dim)).astype(np.float32), "bfloat16")
        k = dim // world
        results = {}
        for name in ROW_PARALLEL[:2]:
            part = torch.from_numpy(oracle_product(sp[name], x[:, rank * k:(rank + 1) * k]))
            dist.all_reduce(part)  # the sum over ranks, as after a row-parallel layer
            results[name] = part.numpy()
            if rank == 0:
                want = oracle_product(parts[name], x)
                results[name + ".rel"] = float(np.linalg.norm(part.numpy() - want) / np.linalg.norm(want))
        out[rank] = results
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_row_parallel_partials_all_reduced_over_gloo():
    world, port = 2, free_port()
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
    for name in ("self_attn.o", "cross_attn.o"):
        assert out[0][name + ".rel"] <= 1e-6
        np.testing.assert_array_equal(out[0][name], out[1][name])  # every rank holds the same sums


def test_random_model_refuses_lowrank_branches_on_shards():
    """svd_rank applies to one stream per GPU: with a tensor-parallel shard the model refuses it before making
    anything (the split's blocks quantize at rank 0)."""
    import pytest
    from wan_dit_lab_b200.generation.causal import random_model
    with pytest.raises(ValueError, match="svd_rank"):
        random_model(num_layers=1, device="cpu", shard=(0, 2), svd_rank=32)
