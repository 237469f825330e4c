"""Benchmark of the quantized-linear hot path on B200.

One step = one ConvRot W8A8 linear over one batch of synthetic activations:
the fused rotate + per-token int8 quantisation kernel followed by the
tcgen05 int8 GEMM with the per-token x per-channel scale, bf16 rounding and
bias epilogue (Int8TensorwiseOps.Linear.forward's compute).

Workload (the ConvRot W8A8 linear configuration): x bf16 [4096, 3072] ~N(0,1)
with 0.1% outlier channels x20, W [12288, 3072] ~N(0, 0.02) rotated and
per-channel int8 quantised once before timing, bias bf16 ~N(0, 0.01),
Hadamard block 128 (Sylvester), seed 1.  The L2 cache is flushed (256 MB
write) before every timed step, outside the timed events.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched with torchrun; every rank runs its own batch (data
parallel over samples, no collective on the data path) and rank 0 prints one
JSON line with the whole-job throughput (max step time over ranks).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "W8A8/W4A8 GEMM TOPS & % INT8 peak; DiT steps/sec at 1/2/4/8 B200"
M, N, K, GROUP, KIND = 4096, 12288, 3072, 128, "sylvester"
SEED = 1
CPU_SAMPLE_ROWS = 4096  # the whole batch: the CPU sample is bounded by time instead
# dram__bytes_read.sum + dram__bytes_write.sum of one GEMM launch at this
# workload, from the ncu capture summarised in profiles/ (None until taken).
GEMM_TRAFFIC_BYTES = 131576832  # ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch (profiles/gemm_i8_pair_w8a8_4096x12288x3072.md)


def load_pkg():
    import __graft_entry__ as ge
    return ge._load_package()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def make_inputs(rows, device, seed=SEED):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K), dtype=np.float32)
    cols = rng.permutation(K)[:max(1, K // 1000)]
    x[:, cols] *= np.float32(20.0)
    w = (np.random.default_rng(1000 + seed).standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    b = np.random.default_rng(2000 + seed).standard_normal(N, dtype=np.float32) * np.float32(0.01)
    xt = torch.from_numpy(x).to(torch.bfloat16)
    wt = torch.from_numpy(w)
    bt = torch.from_numpy(b).to(torch.bfloat16)
    if device is not None:
        xt, wt, bt = xt.to(device), wt.to(device), bt.to(device)
    return xt, wt, bt


_SAMPLER = r"""
import sys, time, pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
while True:
    print(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
          pynvml.nvmlDeviceGetCurrentClocksEventReasons(h), flush=True)
    time.sleep(0.001)
"""


class ClockSampler:
    """SM clock and clock-event (throttle) reasons, sampled through NVML by a
    separate process (read-only queries; a thread would contend for the GIL
    with the launch loop) while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        ids = vis.split(",") if vis else []
        self.nvml_index = int(ids[gpu_index]) if len(ids) > gpu_index and ids[gpu_index].isdigit() else gpu_index
        self.proc, self.lines = None, []

    def __enter__(self):
        import subprocess
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, str(self.nvml_index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.proc.stdout.readline()  # wait until sampling has started
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = out.splitlines()

    def summary(self):
        samples = []
        for ln in self.lines:
            parts = ln.split()
            if len(parts) == 2 and parts[0].isdigit() and parts[1].isdigit():
                samples.append((int(parts[0]), int(parts[1])))
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        try:
            import pynvml
            pynvml.nvmlInit()
            mx = pynvml.nvmlDeviceGetMaxClockInfo(pynvml.nvmlDeviceGetHandleByIndex(self.nvml_index),
                                                  pynvml.NVML_CLOCK_SM)
        except Exception:
            mx = None
        reasons = sorted({k for _, rs in samples for k, bit in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(s for s, _ in samples), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(samples)}


def cpu_baseline(min_seconds=10.0, max_runs=60):
    """The reference's PyTorch CPU path (restated in oracle/torch_cpu_path.py)
    on the workload, all host threads, repeated for about ``min_seconds``."""
    from oracle import torch_cpu_path as R
    torch.set_num_threads(os.cpu_count() or 1)
    x, w, b = make_inputs(CPU_SAMPLE_ROWS, None)
    H = R.hadamard(GROUP, KIND)
    wr = R.rotate_activation(w, H, GROUP)  # rotate_weight: H symmetric
    wq, ws = R.quantize_int8_axiswise(wr, dim=1)
    R.convrot_w8a8_linear(x, H, GROUP, wq, ws, b, torch.bfloat16)  # warm-up
    ts = []
    t_start = time.perf_counter()
    while len(ts) < max_runs and (time.perf_counter() - t_start < min_seconds or len(ts) < 3):
        t0 = time.perf_counter()
        R.convrot_w8a8_linear(x, H, GROUP, wq, ws, b, torch.bfloat16)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    steps = len(ts)
    return {"value": round(2.0 * CPU_SAMPLE_ROWS * N * K / t / 1e12, 4), "unit": "TOPS",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{CPU_SAMPLE_ROWS} of {M} rows, median of {steps} runs "
                      f"({t * 1e3:.1f} ms each); reference PyTorch CPU path (bf16 rotation matmul, "
                      f"torch._int_mm, two-rounding epilogue)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = max(1, args.steps)
    from oracle import torch_cpu_path as R
    torch.set_num_threads(os.cpu_count() or 1)
    x, w, b = make_inputs(CPU_SAMPLE_ROWS, None)
    H = R.hadamard(GROUP, KIND)
    wq, ws = R.quantize_int8_axiswise(R.rotate_activation(w, H, GROUP), dim=1)
    for _ in range(args.warmup):
        R.convrot_w8a8_linear(x, H, GROUP, wq, ws, b, torch.bfloat16)
    t0 = time.perf_counter()
    for _ in range(steps):
        R.convrot_w8a8_linear(x, H, GROUP, wq, ws, b, torch.bfloat16)
    t = (time.perf_counter() - t0) / steps
    v = round(2.0 * CPU_SAMPLE_ROWS * N * K / t / 1e12, 4)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TOPS", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": {"workload": f"convrot_w8a8_linear M={M} N={N} K={K} hadamard={KIND}{GROUP} bf16 "
                                   f"(CPU sample: {CPU_SAMPLE_ROWS} rows per step)", "M": M, "N": N, "K": K},
            "cpu_baseline": {"value": v, "unit": "TOPS", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"{CPU_SAMPLE_ROWS} of {M} rows per step"},
            "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = load_pkg()
    ops = pkg.ops
    rot = (KIND, GROUP)
    x, w, b = make_inputs(M, dev, seed=SEED + rank)
    wq, ws = ops.quant_weight_int8(w, rot)
    del w
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step():
        xq, xs = ops.quant_act_int8(x, rot)
        return xq, xs

    # warm-up runs exactly the timed body, so the caching allocator already
    # holds two output blocks (the previous step's y is alive while the next
    # one is allocated) and no cudaMalloc lands inside a timed step
    y = None
    for _ in range(max(3, args.warmup)):
        xq, xs = ops.quant_act_int8(x, rot)
        y = ops.gemm_w8a8(xq, xs, wq, ws, b, torch.bfloat16)
    torch.cuda.synchronize()

    s = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            # keep the GPU busy while the host enqueues the step, so the
            # events time kernels, not host launch latency
            torch.cuda._sleep(1_000_000)
            ev[i][0].record(s)
            xq, xs = ops.quant_act_int8(x, rot)
            ev[i][1].record(s)
            y = ops.gemm_w8a8(xq, xs, wq, ws, b, torch.bfloat16)
            ev[i][2].record(s)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t_quant = [e[0].elapsed_time(e[1]) for e in ev]
    t_gemm = [e[1].elapsed_time(e[2]) for e in ev]
    t_step = [e[0].elapsed_time(e[2]) for e in ev]
    total_ms = sum(t_step)
    tmax = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(tmax, op=torch.distributed.ReduceOp.MAX)
    total_ms = float(tmax.item())

    # e2e through the public API with host buffers (pinned) every step
    pub = pkg.int8_quant
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        xd = x_host.to(dev, non_blocking=True)
        y_host.copy_(pub.int8_forward_dynamic_per_row(xd, wq, ws, b, torch.bfloat16, rot), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        xd = x_host.to(dev, non_blocking=True)
        y_host.copy_(pub.int8_forward_dynamic_per_row(xd, wq, ws, b, torch.bfloat16, rot), non_blocking=True)
    e1.record(s)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(e2e_ms, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    ops_per_step = 2.0 * M * N * K
    value = world * args.steps * ops_per_step / (total_ms * 1e-3) / 1e12
    hbm_gbs, bf16_tf, src = peaks()
    int8_peak = 2.0 * bf16_tf  # B200 dense int8 rate is twice dense bf16
    gemm_ms = statistics.mean(t_gemm)
    quant_ms = statistics.mean(t_quant)
    gemm_tops = ops_per_step / (gemm_ms * 1e-3) / 1e12
    quant_bytes = M * K * 2 + M * K + M * 4
    quant_gbs = quant_bytes / (quant_ms * 1e-3) / 1e9
    cpu = cpu_baseline() if (rank == 0 and world == 1) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": {"workload": f"convrot_w8a8_linear M={M} N={N} K={K} hadamard={KIND}{GROUP} bf16 in/out, "
                                   f"per-token x per-channel int8, bias; one batch per GPU",
                       "M": M, "N": N, "K": K, "l2": "flushed (256 MB write) before every timed step",
                       "parallelism": f"dp{world} (independent batches, no collective)"},
            "roofline": {"bound": "tensor", "kernel": "gemm_i8_pair_kernel (tcgen05 kind::i8, CTA pair)",
                         "achieved": round(gemm_tops, 1), "peak": round(int8_peak, 1), "unit": "TOPS",
                         "frac": round(gemm_tops / int8_peak, 4), "traffic": GEMM_TRAFFIC_BYTES,
                         "peak_source": f"2 x {src} dense bf16 ({bf16_tf} TFLOP/s) = dense int8"},
            "roofline_quant": {"bound": "hbm", "kernel": "rowquant_pair_kernel (fused Hadamard-128 + int8)",
                               "achieved": round(quant_gbs, 1), "peak": hbm_gbs, "unit": "GB/s",
                               "frac": round(quant_gbs / hbm_gbs, 4), "bytes": quant_bytes,
                               "us": round(quant_ms * 1e3, 2)},
            "gemm_us": round(gemm_ms * 1e3, 2),
            "e2e": {"value": round(world * args.steps * ops_per_step / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOPS",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                    "api": "int8_quant.int8_forward_dynamic_per_row, pinned host x in, y out"},
            "cpu_baseline": cpu,
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
