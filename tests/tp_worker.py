"""One rank of the tensor-parallel tests, launched by test_tensor_parallel.py
as a separate process (RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT in the
environment).

    python tests/tp_worker.py gather   # gloo, CPU: shard layout + interleave
    python tests/tp_worker.py linear   # nccl, one GPU per rank: fused and
                                       # NCCL modes vs the single-GPU GEMM
Exit status 0 when every check passed."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))


def gather_check():
    from conftest import load_package
    tp = load_package().tensor_parallel
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    m, n = 5, 100
    full = torch.arange(m * n, dtype=torch.float32).reshape(m, n)
    start, stop = tp.shard_bounds(n, world, rank)
    per = tp.shard_bounds(n, world, 0)[1]
    local = torch.zeros((m, per))
    local[:, :stop - start] = full[:, start:stop]
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local)
    out = tp.interleave_shards(torch.stack(parts), n)
    ok = torch.equal(out, full)
    dist.destroy_process_group()
    return ok


def linear_check():
    from conftest import load_package
    P = load_package()
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    g = torch.Generator(device="cpu")
    g.manual_seed(7)
    ok = True
    # n = 3080: not a multiple of 8 * world (uneven last shard); n = 1001: rows
    # of the gathered output not 16-byte multiples (padded buffer stride)
    for n in (3080, 1001):
        k = 1024
        w = torch.randn((n, k), generator=g) * 0.02
        bias = (torch.randn((n,), generator=g) * 0.01).to(torch.bfloat16)
        rot = ("regular", 256)
        wq, ws = P.ops.quant_weight_int8(w.to(dev), rot)
        layers = {mode: P.tensor_parallel.ColumnParallelInt8Linear(wq, ws, bias, rot=rot, mode=mode)
                  for mode in ("fused", "nccl")}
        for step, m in enumerate((300, 300, 300, 64)):
            x = (torch.randn((m, k), generator=g) * (1 + step)).to(torch.bfloat16).to(dev)
            xq, xs = P.ops.quant_act_int8(x, rot)
            want = P.ops.gemm_w8a8(xq, xs, wq, ws, bias.to(dev), torch.bfloat16)
            for mode, layer in layers.items():
                got = layer(x)  # read before the layer's next call (the fused output's lifetime)
                if got.shape != want.shape or not torch.equal(got.view(torch.int16), want.view(torch.int16)):
                    print(f"rank {rank} n {n} mode {mode} step {step}: mismatch "
                          f"{(got.float() - want.float()).abs().max().item()}", flush=True)
                    ok = False
        torch.cuda.synchronize()
        layers.clear()
    ok_t = torch.tensor([int(ok)], device=dev)
    dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    return bool(ok_t.item())


if __name__ == "__main__":
    what = sys.argv[1]
    ok = gather_check() if what == "gather" else linear_check()
    sys.exit(0 if ok else 1)
