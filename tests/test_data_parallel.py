"""Data-parallel sharding and host-side failure detection (CPU, gloo ranks).

Faults are made on the host only: a rank's step raises, or a rank exits
between steps; the other ranks must report it at the next status exchange
instead of hanging."""
import os
import socket
import subprocess
import sys

import pytest

from conftest import load_package

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(what, world, timeout=120):
    port = str(_free_port())
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=port, CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "dp_worker.py"), what], env=env))
    codes = []
    try:
        for p in procs:
            codes.append(p.wait(timeout=timeout))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    return codes


def test_shard_bounds_cover_the_batch():
    dp = load_package().data_parallel
    for n in (0, 1, 7, 16, 17):
        for world in (1, 2, 3, 4, 8):
            bounds = [dp.shard_bounds(n, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == n
            assert all(a <= b for a, b in bounds)
            assert all(b0 == a1 for (_, b0), (a1, _) in zip(bounds, bounds[1:]))
            sizes = [b - a for a, b in bounds]
            assert max(sizes) - min(sizes) <= 1
    assert dp.shard_bounds(16, 8, 3) == (6, 8)  # the DiT step: 16 samples, 2 per rank at 8 GPUs
    with pytest.raises(ValueError):
        dp.shard_bounds(4, 2, 2)


def test_steps_succeed_two_ranks():
    assert _run_ranks("ok", 2) == [0, 0]


@pytest.mark.parametrize("world", [2, 3])
def test_step_failure_is_reported_on_every_rank(world):
    assert _run_ranks("raise", world) == [0] * world


def test_lost_rank_is_detected_by_the_survivor():
    # the exiting rank's own status is not checked (it exits with 0 by design)
    codes = _run_ranks("exit", 2)
    assert codes[0] == 0, codes
