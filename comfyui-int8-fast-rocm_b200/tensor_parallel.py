"""Column-parallel (tensor-parallel) W8A8 linear: the single-sample latency
mode across the GPUs of one node.

Every rank of the process group keeps one contiguous block of output
features (rows of the int8 weight, their per-channel scales and bias),
quantises the whole replicated activation, and runs its GEMM shard.  In the
default ``mode="fused"`` the GEMM epilogue stores its output columns straight
into every rank's output buffer -- peer mappings of one torch
symmetric-memory allocation reached over NVLink -- and a device-side barrier
then makes the gathered ``[M, N]`` output visible everywhere: no separate
all-gather pass.  ``mode="nccl"`` computes the shard into a local tensor and
gathers it with ``all_gather_into_tensor`` (the baseline the fused path
replaces).

Lifetime of a fused call's output: it is a view of one of two symmetric
buffers that alternate between calls (rows padded to 16 bytes, so a layer
of any width fits), returned without a copy.  Call k+2 rewrites it, and every
rank's writes of call k+2 come after the device barrier that ends call k+1,
which each rank reaches only after the work it enqueued on its stream
before call k+1.  So the output of call k may be read by any work enqueued
on the calling stream before the layer's next call; clone it to keep it
longer.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from . import ops

SHARD_ALIGN = 8  # output columns per shard boundary: 16 bytes of bf16/f16


def shard_bounds(n: int, world: int, rank: int, align: int = SHARD_ALIGN):
    """[start, stop) of rank's output features: equal blocks rounded up to
    ``align`` columns (16-byte aligned column offsets), the last ranks
    possibly shorter or empty."""
    per = -(-n // world)
    per = -(-per // align) * align
    start = min(n, rank * per)
    return start, min(n, start + per)


def padded_width(n: int, align: int = SHARD_ALIGN) -> int:
    """Row stride of the gathered output buffer: ``n`` rounded up to
    ``align`` columns (the fused kernel stores 16-byte rows)."""
    return -(-n // align) * align


def interleave_shards(gathered: torch.Tensor, n: int) -> torch.Tensor:
    """``[world, M, per]`` shards (zero padded) -> ``[M, n]`` in column
    order."""
    world, m, per = gathered.shape
    return gathered.permute(1, 0, 2).reshape(m, world * per)[:, :n]


class ColumnParallelInt8Linear:
    """W8A8 (+ optional ConvRot) linear with its output features split over
    ``group``.  ``weight_q`` [N, K] int8 and ``weight_scale`` [N] / [N, 1]
    float32 are the full layer (every rank passes the same tensors, e.g. as
    loaded); each rank keeps only its shard on its current CUDA device."""

    def __init__(self, weight_q: torch.Tensor, weight_scale: torch.Tensor, bias=None, group=None, rot=None,
                 out_dtype: torch.dtype = torch.bfloat16, mode: str = "fused"):
        if mode not in ("fused", "nccl"):
            raise ValueError(f"mode must be 'fused' or 'nccl', got {mode!r}")
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("at most 8 ranks (one NVLink domain of a node)")
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.n, self.k = weight_q.shape
        self.start, self.stop = shard_bounds(self.n, self.world, self.rank)
        self.per = shard_bounds(self.n, self.world, 0)[1]
        self.wq = weight_q[self.start:self.stop].to(self.device).contiguous()
        self.ws = weight_scale.reshape(-1)[self.start:self.stop].to(self.device, torch.float32).contiguous()
        self.bias = None if bias is None else \
            bias.reshape(-1)[self.start:self.stop].to(self.device, out_dtype).contiguous()
        self.rot = rot
        self.out_dtype = out_dtype
        self.mode = mode
        self._bufs = {}   # rows -> [(buffer, handle), (buffer, handle)]
        self._calls = 0

    # -- symmetric output buffers ------------------------------------------
    def _buffers(self, m: int):
        got = self._bufs.get(m)
        if got is None:
            import torch.distributed._symmetric_memory as symm_mem
            got = []
            for _ in range(2):
                t = symm_mem.empty((m, padded_width(self.n)), dtype=self.out_dtype, device=self.device)
                h = symm_mem.rendezvous(t, self.group)
                base = h.buffer_ptrs[self.rank]
                ptrs = [p + (t.data_ptr() - base) for p in h.buffer_ptrs]
                got.append((t, h, (ctypes.c_void_p * self.world)(*ptrs)))
            self._bufs[m] = got
        return got

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.forward(x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        m = x2.shape[0]
        xq, xs = ops.quant_act_int8(x2.to(self.out_dtype) if x2.dtype != self.out_dtype else x2, self.rot)
        if self.mode == "nccl":
            y = self._forward_nccl(xq, xs, m)
        else:
            y = self._forward_fused(xq, xs, m)
        return y.reshape(*shape[:-1], self.n)

    def _forward_fused(self, xq, xs, m):
        t, h, ptrs = self._buffers(m)[self._calls & 1]
        self._calls += 1
        if self.stop > self.start:
            N.call("qlin_set_device", self.device.index)
            N.call("qlin_gemm_w8a8_allgather", xq.data_ptr(), xs.data_ptr(), self.wq.data_ptr(),
                   self.ws.data_ptr(), N.WSCALE_ROW, 0 if self.bias is None else self.bias.data_ptr(),
                   ctypes.cast(ptrs, ctypes.c_void_p), self.world, self.start, t.shape[1],
                   ops.dtype_code(self.out_dtype), m, self.stop - self.start, self.k,
                   torch.cuda.current_stream(self.device).cuda_stream)
        h.barrier(channel=0)
        return t[:, :self.n]  # valid until the layer's next call is enqueued (module docstring)

    def _forward_nccl(self, xq, xs, m):
        local = torch.zeros((m, self.per), dtype=self.out_dtype, device=self.device)
        if self.stop > self.start:
            local[:, :self.stop - self.start] = ops.gemm_w8a8(xq, xs, self.wq, self.ws, self.bias, self.out_dtype)
        gathered = torch.empty((self.world, m, self.per), dtype=self.out_dtype, device=self.device)
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        return interleave_shards(gathered, self.n).contiguous()
