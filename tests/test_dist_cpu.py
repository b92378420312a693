"""The bench's multi-replica bookkeeping on CPU: two gloo ranks.

`bench.py --gpus N` runs one replica per GPU and reports the whole-job rate
(every rank's tokens over the slowest rank's device time); the same helpers
run here over gloo with host tensors, so the N > 1 path is checked without a
GPU.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bench.barrier(dist)
        mx = bench.max_over_ranks(dist, float(rank + 1))
        sm = bench.sum_over_ranks(dist, float(10 * (rank + 1)))
        # rank r processed 64 * (r + 1) tokens in (r + 1) * 0.5 s
        val, tmax = bench.job_throughput(dist, 64.0 * (rank + 1), 0.5 * (rank + 1))
        q.put((rank, mx, sm, val, tmax))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_aggregate_like_the_bench():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, mx, sm, val, tmax in res:
        assert mx == 2.0
        assert sm == 30.0
        assert tmax == 1.0                       # the slowest rank's time
        assert val == pytest.approx(192.0 / 1.0)  # (64 + 128) tokens over 1 s
