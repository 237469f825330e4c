"""Packed-INT4 x INT8 GEMM with the reference's triton_int4_mm API
(triton_int4_mm.py:123-170), on tcgen05 tensor cores: the packed weight
slab is TMA-loaded, unpacked to int8 in shared memory and fed to the i8 MMA.

A: int8 [M, K] activations (values normally in [-7, 7]);
W: int8 [N, K // 2] packed signed int4, low nibble = even K column.
"""
from __future__ import annotations

import torch

from . import library as kops  # the kernels as registered torch.library operators


def triton_int4_mm(a: torch.Tensor, packed_weight: torch.Tensor, out_dtype: torch.dtype = torch.int32) -> torch.Tensor:
    """a[M,K] @ unpack(packed_weight[N,K/2]).T -> [M,N] (int32)."""
    assert a.ndim == 2
    assert packed_weight.ndim == 2
    assert a.dtype == torch.int8
    assert packed_weight.dtype == torch.int8
    assert a.device == packed_weight.device
    assert a.is_contiguous(), "Matrix A must be contiguous"
    M, K = a.shape
    N, K_packed = packed_weight.shape
    assert K == K_packed * 2, f"K mismatch: activation K={K}, packed weight represents {K_packed * 2}"
    assert K % 2 == 0
    c = kops.int4_mm(a, packed_weight)
    return c if out_dtype == torch.int32 else c.to(out_dtype)
