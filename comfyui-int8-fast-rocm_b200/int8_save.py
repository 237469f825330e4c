"""Writing quantised models back to disk in the formats the loaders read.

``quantized_state_dict`` walks a model and emits, for every quantised
``Int8TensorwiseOps.Linear`` / ``Int4ConvRotOps.Linear``, its stored weight
and scale tensors plus the per-layer ``comfy_quant`` marker (the layer's
JSON description as uint8 bytes) that the reference's save node writes
(int8_save.py:219-256):

* INT8 layers: ``{"format": "int8_tensorwise", "convrot": bool,
  "convrot_groupsize": g (with ConvRot), "per_row": bool}``, the int8
  ``weight`` [N, K] and ``weight_scale`` ([N, 1] per row, [1] tensor-wide);
* INT4 layers: ``{"format": "convrot_w4a4", "convrot_groupsize": g,
  "linear_dtype": "int4"}`` with the packed ``weight`` [N, K/2] and
  ``weight_scale`` [N]; an int8 layer inside an INT4 model is written in
  the INT8 format above;
* every other parameter and buffer as it is.

Loading the result through the same custom operations restores the layers
bit for bit (tests/test_saver.py).  ``save_quantized`` writes the dict to a
safetensors file.  Only the on-disk format is implemented here; the
reference's ComfyUI save node (LoRA materialisation, CLIP saving) is not.
"""
from __future__ import annotations

import json

import torch


def comfy_quant_tensor(conf: dict) -> torch.Tensor:
    """A layer's ``comfy_quant`` marker: its JSON description as uint8 bytes."""
    return torch.frombuffer(bytearray(json.dumps(conf).encode("utf-8")), dtype=torch.uint8)


def layer_quant_conf(module):
    """The ``comfy_quant`` description of a quantised linear layer, or None
    for a layer kept in its original precision."""
    if not getattr(module, "_is_quantized", False):
        return None
    if getattr(module, "_is_w4a8", False):
        raise NotImplementedError("asym_w4a8_int8 layers are loaded from their own checkpoints, not re-saved")
    if getattr(module, "_linear_dtype", "int8_tensorwise") == "int4":
        return {"format": "convrot_w4a4", "convrot_groupsize": int(module._convrot_groupsize), "linear_dtype": "int4"}
    conf = {"format": "int8_tensorwise", "convrot": bool(getattr(module, "_use_convrot", False))}
    if conf["convrot"]:
        conf["convrot_groupsize"] = int(module._convrot_groupsize)
    conf["per_row"] = bool(getattr(module, "_is_per_row", False))
    return conf


def _scale_for_disk(module, conf):
    s = module.weight_scale.detach().float().cpu()
    if conf["format"] == "convrot_w4a4":
        return s.reshape(-1).contiguous()
    return s.reshape(-1, 1).contiguous() if conf["per_row"] else s.reshape(1).contiguous()


def quantized_state_dict(model: torch.nn.Module, prefix: str = "") -> dict:
    """State dict of ``model`` with every quantised linear in its on-disk
    format (see the module docstring); keys are ``prefix`` + module path."""
    out = {}
    handled = set()
    for name, module in model.named_modules():
        conf = layer_quant_conf(module)
        if conf is None:
            continue
        base = prefix + (name + "." if name else "")
        out[base + "weight"] = module.weight.detach().cpu().contiguous()
        out[base + "weight_scale"] = _scale_for_disk(module, conf)
        out[base + "comfy_quant"] = comfy_quant_tensor(conf)
        if module.bias is not None:
            out[base + "bias"] = module.bias.detach().cpu().contiguous()
        handled.update(base + k for k in ("weight", "weight_scale", "bias"))
    for key, t in model.state_dict().items():
        k = prefix + key
        if k not in handled and t is not None:
            out[k] = t.detach().cpu().contiguous()
    return out


def save_quantized(model: torch.nn.Module, path: str, prefix: str = "", metadata=None) -> dict:
    """Write :func:`quantized_state_dict` to a safetensors file; returns it."""
    from safetensors.torch import save_file

    sd = quantized_state_dict(model, prefix)
    save_file(sd, path, metadata=metadata)
    return sd
