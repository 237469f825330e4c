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
consumes (int8_quant.py:679-687) in one pass.
"""
from __future__ import annotations

import json
import logging

import torch
from torch import Tensor

from . import ops


def unpack_int4_unsigned(packed: Tensor) -> Tensor:
    """[N, K//2] int8 -> [N, K] int32 codes in [0, 15] (w4a8_int8.py:29-43)."""
    assert packed.ndim == 2, f"Expected 2D tensor, got {packed.ndim}D"
    p32 = packed.to(torch.int32) & 0xFF
    return torch.stack([p32 & 0x0F, (p32 >> 4) & 0x0F], dim=-1).reshape(packed.shape[0], -1)


def requant_int8(packed: Tensor, codebook: Tensor, s_channel: Tensor, s_rel: Tensor, group_size: int):
    """Fused dequant -> quantize_int8_axiswise(dim=1): (int8 [N,K], f32 [N,1])."""
    return ops.requant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size)


def dequant_asym_w4a8_to_float(packed_codes: Tensor, codebook: Tensor, s_channel: Tensor, s_rel: Tensor,
                               group_size: int) -> Tensor:
    """float32 [N, K] dequantised weight (w4a8_int8.py:46-75).  A format
    utility off the hot path (diagnostics, LoRA baking): element-wise torch
    on the weight's device, same expression order as the reference."""
    N, K_packed = packed_codes.shape
    K = K_packed * 2
    codes = unpack_int4_unsigned(packed_codes)
    vals = codebook.to(torch.float32)[codes.long()]
    s_rel_f32 = s_rel.to(torch.float32)
    if s_rel_f32.shape[1] * group_size != K:
        raise ValueError(
            f"W4A8: group mismatch, num_groups({s_rel_f32.shape[1]}) * group_size({group_size}) != K({K})")
    return vals * s_channel.to(torch.float32).reshape(N, 1) * s_rel_f32.repeat_interleave(group_size, dim=1)


def bridge_w4a8_metadata_to_comfy_quant(state_dict: dict, metadata) -> int:
    """Copy per-layer ``asym_w4a8_int8`` entries of the safetensors header's
    ``_quantization_metadata`` into ``<layer>.comfy_quant`` marker tensors
    (w4a8_int8.py:78-121)."""
    if not metadata or "_quantization_metadata" not in metadata:
        return 0
    try:
        quant_meta = json.loads(metadata["_quantization_metadata"])
    except Exception as e:
        logging.warning(f"W4A8: failed to parse _quantization_metadata: {e}")
        return 0
    bridged = 0
    for layer_name, conf in quant_meta.get("layers", {}).items():
        if conf.get("format") != "asym_w4a8_int8":
            continue
        candidates = (layer_name + ".weight", "model." + layer_name + ".weight",
                      "diffusion_model." + layer_name + ".weight", "model.diffusion_model." + layer_name + ".weight")
        weight_key = next((k for k in candidates if k in state_dict), None)
        if weight_key is None:
            suffix = layer_name + ".weight"
            matches = [k for k in state_dict if k == suffix or k.endswith("." + suffix)]
            if len(matches) == 1:
                weight_key = matches[0]
        if weight_key is None:
            logging.warning(f"W4A8: metadata bridge could not find weight for layer '{layer_name}'")
            continue
        quant_key = weight_key[:-len(".weight")] + ".comfy_quant"
        if quant_key not in state_dict:
            payload = json.dumps(conf, separators=(",", ":")).encode("utf-8")
            state_dict[quant_key] = torch.tensor(list(payload), dtype=torch.uint8)
        bridged += 1
    if bridged:
        logging.info(f"W4A8: bridged safetensors header metadata for {bridged} asym_w4a8_int8 layers")
    return bridged
