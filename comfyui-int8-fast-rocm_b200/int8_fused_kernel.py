"""Module-level kernel API of the reference's int8_fused_kernel.py, backed by
the sm_100a kernels (the names are kept so existing imports work).

Numerics follow the reference's PyTorch path (int8_quant.py:41-52,
137-164), not its Triton rounding: codes are ``rint(x * (1/scale))``
(round-half-even) and the epilogue rounds to the output dtype before adding
the bias.  That is what the reference produces on CPU.
"""
from __future__ import annotations

import torch

from . import library as kops  # the kernels as registered torch.library operators


def triton_quantize_rowwise(x: torch.Tensor):
    """[rows, cols] float -> (int8 [rows, cols], float32 [rows, 1])
    (int8_fused_kernel.py:67-85)."""
    return kops.quant_act_int8(x)


def _linear(x, weight, weight_scale, bias, compute_dtype, x_q, per_row):
    shape = x.shape
    if x_q is None:
        x_int8, x_scale = kops.quant_act_int8(x.reshape(-1, shape[-1]))
    else:
        x_int8, x_scale = x_q
    n = weight.shape[0]
    if not isinstance(weight_scale, torch.Tensor):
        weight_scale = torch.tensor([float(weight_scale)], dtype=torch.float32, device=x_int8.device)
    out = kops.gemm_w8a8(x_int8, x_scale, weight.to(x_int8.device), weight_scale, bias, compute_dtype,
                        per_row=per_row)
    return out.reshape(tuple(shape[:-1]) + (n,))


def triton_int8_linear(x, weight, weight_scale, bias=None, compute_dtype=torch.float16, x_q=None):
    """W8A8 linear with a scalar weight scale (int8_fused_kernel.py:184-244;
    epilogue order of int8_forward_dynamic, int8_quant.py:113-133).  A
    per-channel scale tensor selects the per-row epilogue."""
    ws = weight_scale
    per_row = isinstance(ws, torch.Tensor) and ws.numel() > 1
    return _linear(x, weight, ws, bias, compute_dtype, x_q, per_row)


def triton_int8_linear_per_row(x, weight, weight_scale, bias=None, compute_dtype=torch.float16, x_q=None):
    """W8A8 linear with per-output-channel weight scales [N,1]
    (int8_fused_kernel.py:332-377; epilogue order of
    int8_forward_dynamic_per_row, int8_quant.py:137-164)."""
    return _linear(x, weight, weight_scale, bias, compute_dtype, x_q, True)


def triton_situ(x: torch.Tensor) -> torch.Tensor:
    """[..., 2K] ([hidden | gate]) -> [..., K] SiTU activation
    (int8_fused_kernel.py:389-440)."""
    return kops.situ(x)
