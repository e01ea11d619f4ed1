"""The multi-GPU bench path on CPU: replicas, one process per rank, over a gloo group.

Batch-1 decode does not shard (multi-GPU means independent replicas): each rank runs its own
model copy and the job reports the slowest rank's time for all ranks' tokens. These tests run
that aggregation with world size 2 on the gloo backend, and the reference arm's rank rule.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _replica(rank, world, port, times, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        slowest = bench.max_over_ranks(times[rank], dist, torch.device("cpu"))
        out[rank] = (slowest, bench.job_throughput(world, 64, slowest))
    finally:
        dist.destroy_process_group()


def test_slowest_rank_sets_the_job_time():
    world, port = 2, free_port()
    times = [0.050, 0.080]
    out = mp.Manager().dict()
    mp.spawn(_replica, args=(world, port, times, out), nprocs=world, join=True)
    for rank in range(world):
        slowest, tput = out[rank]
        assert slowest == max(times)
        assert abs(tput - world * 64 / max(times)) < 1e-9


def test_single_process_needs_no_group():
    assert bench.max_over_ranks(0.25, None, torch.device("cpu")) == 0.25
    assert bench.job_throughput(1, 10, 0.5) == 20.0


def test_reference_arm_prints_on_rank_zero_only():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], env=env, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0
    assert res.stdout.strip() == ""
