"""The reference's PyTorch CPU branch of the W8A8 ConvRot linear, restated
with the same torch calls -- TEST AND CPU-REFERENCE-ARM INFRASTRUCTURE ONLY.

This is what the reference runs when the activation is on the CPU
(int8_quant.py:148-164 with rotate_activation, convrot.py:89-118, and
quantize_int8_axiswise, int8_quant.py:41-52): a bf16 batched matmul for the
rotation, element-wise quantisation, ``torch._int_mm`` (oneDNN int8 on CPU)
and the two-rounding epilogue.  ``bench.py`` times it on the host cores as the
CPU baseline (``--impl reference`` and the ``cpu_baseline`` field); the tests
check that it agrees with the numpy oracle.  The product never imports it.
"""
from __future__ import annotations

import torch


def hadamard(size: int, kind: str) -> torch.Tensor:
    """Normalised Hadamard as built by convrot.build_hadamard (regular) or
    ``scipy.linalg.hadamard(size) / size**0.5`` (Sylvester), float32."""
    if kind == "regular":
        h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float32)
        h = h4
        while h.shape[0] < size:
            h = torch.kron(h, h4)
    else:
        h = torch.ones((1, 1), dtype=torch.float32)
        while h.shape[0] < size:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / (size ** 0.5)


def rotate_activation(x: torch.Tensor, H: torch.Tensor, group: int) -> torch.Tensor:
    """convrot.py:89-118."""
    shp = x.shape
    xg = x.view(*shp[:-1], shp[-1] // group, group)
    return torch.matmul(xg, H.to(dtype=x.dtype)).view(shp)


def quantize_int8_axiswise(x: torch.Tensor, dim: int):
    """int8_quant.py:41-52."""
    abs_max = x.abs().amax(dim=dim, keepdim=True)
    scale = (abs_max.float() / 127.0).clamp(min=1e-30)
    q = x.float().mul(1.0 / scale).round_().clamp_(-128.0, 127.0).to(torch.int8)
    return q, scale


@torch.no_grad()
def int8_forward_dynamic_per_row(x, weight, weight_scale, bias, compute_dtype):
    """int8_quant.py:148-164 (CPU branch)."""
    x_8, x_scale = quantize_int8_axiswise(x, dim=-1)
    res = torch._int_mm(x_8, weight.T)
    res_scaled = res.float().mul_(x_scale).mul_(weight_scale.T).to(compute_dtype)
    if bias is not None:
        res_scaled = res_scaled + bias.to(compute_dtype)
    return res_scaled


@torch.no_grad()
def convrot_w8a8_linear(x, H, group, weight, weight_scale, bias, compute_dtype):
    """Int8TensorwiseOps.Linear.forward's compute for a ConvRot layer
    (int8_quant.py:697-716) on CPU tensors."""
    x_2d = x.reshape(-1, x.shape[-1]).to(compute_dtype)
    if H is not None:
        x_2d = rotate_activation(x_2d, H, group)
    return int8_forward_dynamic_per_row(x_2d, weight, weight_scale, bias, compute_dtype)
