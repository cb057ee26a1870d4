"""The multi-rank (replica) bookkeeping of bench.py on CPU with two gloo ranks: every rank
contributes its timed duration, the job's time is the slowest rank's, and the whole-job rate
counts every rank's units; the reference arm runs on rank 0 only."""
import os
import socket
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, out):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ms = [120.0, 150.0][rank]  # rank 1 is the slower replica
        ms_max = bench.max_over_ranks(ms, world, device="cpu")
        out[rank] = (ms_max, bench.job_rate(256, world, ms_max / 1000.0))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_slowest_replica():
    world = 2
    out = mp.Manager().dict()
    mp.spawn(worker, args=(world, free_port(), out), nprocs=world, join=True)
    for r in range(world):
        ms_max, rate = out[r]
        assert ms_max == 150.0  # every rank sees the slowest rank's time
        assert rate == pytest.approx(2 * 256 / 0.150)


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.max_over_ranks(12.5, 1) == 12.5
    assert bench.job_rate(10, 1, 2.0) == 5.0


def test_reference_arm_runs_on_rank_zero_only():
    sys.path.insert(0, ROOT)
    import argparse

    import bench

    args = argparse.Namespace(gpus=2, steps=2, warmup=1)
    assert bench.run_reference_arm(args, rank=1, world=2) == 0  # no work, no output on rank 1
