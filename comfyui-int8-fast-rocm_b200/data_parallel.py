"""Data-parallel sharding of batch work over the GPUs of one node, with
failure detection on the host between steps.

The quantised-linear path shards by sample (or CFG branch): every rank holds
a full replica of the int8 weights and runs its own contiguous slice of the
batch, with no collective on the data path.  The only cross-rank traffic is
a status exchange after each step:

* every rank calls :meth:`StepMonitor.check` after each step, also when its
  step raised, so all ranks take the same collective in the same order;
* a rank whose step raised reports it there; every rank then raises
  :class:`RankFailure` naming the failed ranks and the step (the failed rank
  chains its own exception);
* a rank that exited or stopped answering makes the exchange itself fail
  (connection closed, or the process group's timeout); the survivors raise
  :class:`RankFailure` with ``ranks=None``.

Nothing here touches a kernel in flight: a rank leaves only between steps.
The reference node pack has no multi-GPU path; this module serves the
sharded DiT step of the benchmark and any host that runs several GPUs.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

__all__ = ["RankFailure", "shard_bounds", "shard_slice", "StepMonitor"]


class RankFailure(RuntimeError):
    """A step failed on one or more ranks (``ranks``), or a rank was lost
    (``ranks`` is None) before step ``step`` completed."""

    def __init__(self, step: int, ranks: Optional[List[int]], reason: str):
        self.step = step
        self.ranks = ranks
        self.reason = reason
        who = "a rank was lost" if ranks is None else f"rank(s) {ranks} failed"
        super().__init__(f"step {step}: {who}: {reason}")


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous slice [start, stop) of n samples owned by `rank`; the first
    n % world ranks take one sample more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n < 0:
        raise ValueError("negative sample count")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_slice(batch: Sequence, world: int, rank: int):
    """This rank's part of `batch` (anything sliceable along its first axis)."""
    start, stop = shard_bounds(len(batch), world, rank)
    return batch[start:stop]


class StepMonitor:
    """Status exchange between data-parallel steps.

    ``check(step, error)`` all-gathers one int per rank (0 = the step
    succeeded); ``run(step_fn, steps)`` calls ``step_fn(i)`` and checks
    after each step.  ``device`` is where the status tensor lives: the
    rank's GPU for NCCL, the CPU for gloo."""

    def __init__(self, group=None, device: Optional[torch.device] = None):
        if not dist.is_initialized():
            raise RuntimeError("StepMonitor needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if device is None:
            backend = dist.get_backend(group)
            device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
        self.device = device

    def check(self, step: int, error: Optional[BaseException] = None) -> None:
        status = torch.tensor([0 if error is None else 1], dtype=torch.int32, device=self.device)
        parts = [torch.empty_like(status) for _ in range(self.world)]
        try:
            dist.all_gather(parts, status, group=self.group)
        except Exception as e:  # a peer exited or timed out: the exchange itself failed
            raise RankFailure(step, None, f"status exchange failed ({type(e).__name__}: {e})") from (error or e)
        failed = [r for r, t in enumerate(parts) if int(t.item()) != 0]
        if failed:
            reason = repr(error) if error is not None else "see the failed rank's log"
            raise RankFailure(step, failed, reason) from error

    def run(self, step_fn: Callable[[int], object], steps: int, first_step: int = 0) -> list:
        """Run `steps` steps, checking status after each; returns the
        step results of this rank."""
        out = []
        for i in range(first_step, first_step + steps):
            err = None
            try:
                out.append(step_fn(i))
            except Exception as e:  # reported to every rank by the exchange below
                err = e
            self.check(i, err)
        return out
