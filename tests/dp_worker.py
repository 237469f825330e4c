"""One rank of the data-parallel failure-detection tests, launched by
test_data_parallel.py as a separate process over gloo on the CPU (RANK /
WORLD_SIZE / MASTER_ADDR / MASTER_PORT in the environment).

    python tests/dp_worker.py ok      # every step succeeds on every rank
    python tests/dp_worker.py raise   # the last rank raises in step 2
    python tests/dp_worker.py exit    # the last rank exits before step 2

Exit status 0 when this rank observed what the scenario expects."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))


def main(what):
    from conftest import load_package
    dp = load_package().data_parallel
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    rank, world = dist.get_rank(), dist.get_world_size()
    mon = dp.StepMonitor()
    last = world - 1
    samples = torch.arange(16)
    mine = dp.shard_slice(samples, world, rank)

    def step(i):
        if what == "raise" and rank == last and i == 2:
            raise ValueError("injected step failure")
        if what == "exit" and rank == last and i == 2:
            os._exit(0)  # leaves between steps: nothing in flight
        return int(mine.sum()) + i

    try:
        out = mon.run(step, 4)
    except dp.RankFailure as e:
        if what == "raise":
            ok = e.step == 2 and e.ranks == [last]
            if rank == last:
                ok = ok and isinstance(e.__cause__, ValueError)
        else:
            ok = what == "exit" and rank != last and e.step == 2 and e.ranks is None
        print(f"rank {rank}: {e}", flush=True)
        return ok
    ok = what == "ok" and len(out) == 4
    total = torch.tensor([out[0]])
    dist.all_reduce(total)
    ok = ok and int(total.item()) == int(samples.sum())
    dist.destroy_process_group()
    return ok


if __name__ == "__main__":
    sys.exit(0 if main(sys.argv[1]) else 1)
