"""The end-to-end bench pipeline's copy/launch schedule (`bench.e2e_schedule`),
simulated on the CPU under random copy and kernel durations.

Model: three in-order streams (upload, compute, download).  A copy starts
when its stream is free and its waited events are done.  A decode launch
follows programmatic dependent launch: it may start once the previous
launch has started and its own waited events are done, reads the step's
seq_lens (staging buffer) right away, and touches the rest of its data only
after the previous launch has finished.  Checked for every step: its upload
lands before its launch starts, a staging buffer is rewritten only after the
launch that read it finished, an output buffer is rewritten only after the
download of its previous content finished, a download starts after its
launch finished, and every waited event was recorded earlier in issue order
(a requirement of stream capture).
"""
from __future__ import annotations

import random

import pytest

import bench


def simulate(ops, group, rng, copy_max=12.0):
    nb = 2 * group
    t_free = {"upload": 0.0, "kernel": 0.0, "download": 0.0}
    start, end = {}, {}
    launch, data = {}, {}
    prev_launch = prev_end = None
    issued = set()
    for op, j, deps in ops:
        for d in deps:
            assert d in issued, f"{op} {j} waits for {d} before it is recorded"
        ready = max([end[d] for d in deps], default=0.0)
        if op == "kernel":
            t0 = max(ready, prev_launch if prev_launch is not None else 0.0)
            t_data = max(t0, prev_end if prev_end is not None else 0.0)
            dur = rng.uniform(5.0, 40.0)
            launch[j], data[j] = t0, t_data
            start[(op, j)], end[(op, j)] = t0, t_data + dur
            prev_launch, prev_end = t0, t_data + dur
        else:
            t0 = max(ready, t_free[op])
            dur = rng.uniform(0.5, copy_max)
            start[(op, j)], end[(op, j)] = t0, t0 + dur
            t_free[op] = t0 + dur
        issued.add((op, j))
    n = len(launch)
    for j in range(n):
        assert end[("upload", j)] <= launch[j], f"step {j}: launch before its upload landed"
        assert start[("download", j)] >= end[("kernel", j)], f"step {j}: download before its kernel ended"
        k = j - nb
        if k >= 0:
            assert start[("upload", j)] >= end[("kernel", k)], f"step {j}: staging rewritten under kernel {k}"
            assert data[j] >= end[("download", k)], f"step {j}: output rewritten before download {k} ended"


@pytest.mark.parametrize("group", [1, 2, 4, 8])
def test_e2e_schedule_is_race_free(group):
    rng = random.Random(group)
    for _ in range(200):
        n = rng.randint(1, 5 * group + 7)
        ops = bench.e2e_schedule(n, group)
        assert sorted((op, j) for op, j, _ in ops) == sorted((op, j) for op in ("upload", "kernel", "download")
                                                               for j in range(n))
        simulate(ops, group, rng)
        simulate(ops, group, rng, copy_max=300.0)  # copies far slower than the kernels


def test_simulation_catches_a_missing_download_wait():
    """Planted mistake: leaders that do not wait for the downloads of the
    output buffers they reuse rewrite an output still being copied out."""
    caught = False
    for seed in range(200):
        rng = random.Random(seed)
        ops = [(op, j, [d for d in deps if d[0] != "download"]) if op == "kernel" else (op, j, deps)
               for op, j, deps in bench.e2e_schedule(40, 4)]
        try:
            simulate(ops, 4, rng, copy_max=300.0)
        except AssertionError as e:
            assert "output rewritten" in str(e)
            caught = True
            break
    assert caught
