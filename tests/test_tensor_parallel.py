"""Column-parallel W8A8 linear: shard layout on CPU (gloo, two ranks) and the
fused GEMM + all-gather against the single-GPU GEMM on two GPUs (nccl)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import cuda_ok, load_package

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(what, world, timeout):
    port = str(_free_port())
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=port, NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), what], env=env))
    codes = []
    try:
        for p in procs:
            codes.append(p.wait(timeout=timeout))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    return codes


def test_shard_bounds():
    tp = load_package().tensor_parallel
    for n in (8, 100, 3072, 3080, 12288):
        for world in (1, 2, 3, 4, 8):
            bounds = [tp.shard_bounds(n, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == n
            for (a0, b0), (a1, b1) in zip(bounds, bounds[1:]):
                assert b0 == a1 and (a1 % 8 == 0 or a1 == n)  # empty trailing shards start at n
            assert all(b >= a for a, b in bounds)


def test_padded_width():
    tp = load_package().tensor_parallel
    assert [tp.padded_width(n) for n in (1, 8, 1001, 3072, 3080)] == [8, 8, 1008, 3072, 3080]


def test_gather_layout_two_ranks_gloo():
    assert _run_ranks("gather", 2, timeout=120) == [0, 0]


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok() or torch.cuda.device_count() < 2, reason="needs two CUDA devices")
def test_column_parallel_linear_two_gpus():
    assert _run_ranks("linear", 2, timeout=300) == [0, 0]
