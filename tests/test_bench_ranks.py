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


def _rank_that_may_die(rank, world, port, out):
    import datetime
    import time
    sys.path.insert(0, str(ROOT))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)  # leaves between steps, before the collective that times the run
    t0 = time.monotonic()
    try:
        bench.combine_ranks(dist, [1.0, 2.0], "cpu")
        out[rank] = ("no error", time.monotonic() - t0)
    except Exception as error:  # noqa: BLE001 - the error the surviving rank must see
        out[rank] = (type(error).__name__, time.monotonic() - t0)


def test_a_rank_that_dies_ends_the_others_collective_with_an_error():
    """Failure detection on the host, as the multi-GPU runs rely on it: a rank that exits between steps makes the
    next collective of the others (the max over ranks of the step times) fail with an error within the process
    group's timeout instead of hanging."""
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = free_port()
    procs = [ctx.Process(target=_rank_that_may_die, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    assert procs[1].exitcode == 3
    assert 0 in out, "the surviving rank recorded nothing"
    kind, waited = out[0]
    assert kind != "no error" and waited < 60, out[0]
