"""Asymmetric W4A8 weight format (format="asym_w4a8_int8"; reference:
w4a8_int8.py).

Tensor layout per layer:
    weight            int8  [N, K//2]  unsigned 4-bit codes, low nibble = even k
    weight_codebook   f32   [16]       Lloyd-Max levels
    weight_s_channel  f32   [N]        per-output-channel scale
    weight_s_rel      f8e4m3 [N, K//group_size] per-group relative scale
    w[n,k] = codebook[code[n,k]] * s_channel[n] * s_rel[n, k // group_size]

The hot path never materialises the float32 weight: ``requant_int8`` fuses
the dequantisation with the per-channel int8 requantisation the W8A8 GEMM
consumes (int8_quant.py:679-687) in one pass.  ``dequant_asym_w4a8_to_float``
runs the same kernel's dequantisation alone.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import library as kops
from .loader_common import bridge_header_quant_metadata


def unpack_int4_unsigned(packed: Tensor) -> Tensor:
    """[N, K//2] int8 -> [N, K] int32 codes in [0, 15] (w4a8_int8.py:29-43)."""
    assert packed.ndim == 2, f"Expected 2D tensor, got {packed.ndim}D"
    p32 = packed.to(torch.int32) & 0xFF
    return torch.stack([p32 & 0x0F, (p32 >> 4) & 0x0F], dim=-1).reshape(packed.shape[0], -1)


def requant_int8(packed: Tensor, codebook: Tensor, s_channel: Tensor, s_rel: Tensor, group_size: int):
    """Fused dequant -> quantize_int8_axiswise(dim=1): (int8 [N,K], f32 [N,1])."""
    return kops.requant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size)


def dequant_asym_w4a8_to_float(packed_codes: Tensor, codebook: Tensor, s_channel: Tensor, s_rel: Tensor,
                               group_size: int) -> Tensor:
    """float32 [N, K] dequantised weight (w4a8_int8.py:46-75): the asym W4A8
    kernel's dequantisation, (codebook[code] * s_channel) * s_rel in float32,
    without the int8 requantisation.  CUDA tensors."""
    return kops.dequant_asym_w4a8(packed_codes, codebook, s_channel, s_rel, group_size)


def bridge_w4a8_metadata_to_comfy_quant(state_dict: dict, metadata) -> int:
    """``<layer>.comfy_quant`` markers for the ``asym_w4a8_int8`` layers listed
    in the safetensors header (w4a8_int8.py:78-121); see
    :func:`loader_common.bridge_header_quant_metadata`."""
    return bridge_header_quant_metadata(state_dict, metadata, ("asym_w4a8_int8",), "asym W4A8")
