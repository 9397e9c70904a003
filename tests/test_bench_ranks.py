"""The multi-GPU path of bench.py on CPU: two gloo ranks, each timing its own replica, combine their durations
as the max over ranks and report the whole job's throughput (weak scaling: every rank processes the same work).
The reference arm runs on rank 0 only."""

import io
import os
import socket
import sys
from contextlib import redirect_stdout
from pathlib import Path

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        step, e2e = bench.combine_ranks(dist, [1.0 + rank, 5.0 - rank], "cpu")
        out[rank] = (step, e2e, bench.job_rate(world, 21, step))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_max_and_sum_the_work():
    world, port = 2, free_port()
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
    for rank in range(world):
        step, e2e, rate = out[rank]
        assert step == 2.0 and e2e == 5.0  # the slowest rank's durations, on every rank
        assert rate == world * 21 / 2.0


def test_reference_arm_prints_on_rank_zero_only():
    sys.path.insert(0, str(ROOT))
    import bench

    class Args:
        workload, steps, warmup, gpus = "linear", 1, 0, 2

    buf = io.StringIO()
    with redirect_stdout(buf):
        assert bench.reference_arm(Args, rank=1, world=2) is None
    assert buf.getvalue() == ""
    assert torch.get_num_threads() >= 1
