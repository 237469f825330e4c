"""ComfyUI glue shared by the INT8 and INT4 ``Linear`` custom operations.

Both classes keep ComfyUI's module protocol (``manual_cast.Linear``
construction, ``set_weight`` / ``set_bias`` for the model patcher, the
low-VRAM weight-function protocol, the float path for layers left
unquantised); the helpers here implement it once.  ComfyUI modules are
passed in by the callers, which define their classes only when ComfyUI is
importable.
"""
from __future__ import annotations

import torch
from torch import nn
import torch.nn.functional as F


def init_linear(module, ops_cls, base_init, in_features, out_features, bias, device, dtype):
    """``Linear.__init__``: while ``ops_cls.skeleton_meta_init`` is set (the
    loaders build a weightless skeleton to map LoRA keys) the parameters
    are meta tensors; otherwise ComfyUI's own constructor runs."""
    if not getattr(ops_cls, "skeleton_meta_init", False):
        base_init(in_features, out_features, bias, device, dtype)
        return
    nn.Module.__init__(module)
    module.in_features, module.out_features = in_features, out_features
    meta = dict(device="meta", **({} if dtype is None else {"dtype": dtype}))
    module.weight = nn.Parameter(torch.empty((out_features, in_features), **meta), requires_grad=False)
    module.bias = nn.Parameter(torch.empty((out_features,), **meta), requires_grad=False) if bias else None


def calc_weight_entries(grouped, default_strength):
    """Loader-grouped pre-LoRA patches ``(value, offset, function[, strength])``
    as the ``(strength, value, strength_model, offset, function)`` entries
    ``comfy.lora.calculate_weight`` takes; three-field entries use
    ``default_strength``."""
    def entry(p):
        value, offset, function = p[0], p[1], p[2]
        return (p[3] if len(p) == 4 else default_strength, value, 1.0, offset, function)
    return [entry(p) for p in grouped or ()]


def store_param(module, name, value, inplace_update, return_weight, inplace_creates=False):
    """``set_weight`` / ``set_bias`` tail: hand the value back, copy it into
    the existing parameter, or install it as a new frozen parameter.  An
    in-place update of a parameter the module lacks is dropped, or with
    ``inplace_creates`` installs it (the INT4 layer's bias behaviour)."""
    if return_weight:
        return value
    current = getattr(module, name)
    if inplace_update and current is not None:
        current.data.copy_(value)
    elif not inplace_update or inplace_creates:
        setattr(module, name, nn.Parameter(value, requires_grad=False))
    return None


def float_forward(module, x, need_cast, cast_bias_weight, uncast_bias_weight):
    """A layer left in its original precision: ComfyUI's cast path when the
    patcher attached weight functions or casting, else the parameters moved
    to the input's device and dtype."""
    if need_cast:
        weight, bias, stream = cast_bias_weight(module, x, offloadable=True)
        y = F.linear(x, weight, bias)
        uncast_bias_weight(module, weight, bias, stream)
        return y
    weight, bias = module.weight, module.bias
    if weight.device != x.device or weight.dtype != x.dtype:
        weight = weight.to(device=x.device, dtype=x.dtype)
        bias = None if bias is None else bias.to(device=x.device, dtype=x.dtype)
    return F.linear(x, weight, bias)


def scale_layout(scale, per_row_hint):
    """A checkpoint's ``weight_scale`` as (float32 buffer, per-row flag): a
    [N, 1] column is per-row, one element (or a plain number) is
    tensor-wide, any other shape is kept as stored and treated as
    tensor-wide; a ``per_row`` entry in the layer's ``comfy_quant`` overrides
    the guess."""
    if not isinstance(scale, torch.Tensor):
        buf, guess = torch.tensor([float(scale)]), False
    elif scale.numel() == 1:
        buf, guess = scale.float().reshape(1), False
    else:
        buf, guess = scale.float(), scale.dim() == 2 and scale.shape[1] == 1
    return buf, guess if per_row_hint is None else bool(per_row_hint)


class QuantLowVramPatch:
    """ComfyUI's low-VRAM weight-function protocol for a quantised layer:
    the patcher calls ``prepare`` before streaming the weight in, the
    instance with the streamed weight, then ``clear_prepared``.  Subclasses
    implement ``apply(weight, patches)``, which patches in float and
    requantises."""
    is_lowvram_patch = True

    def __init__(self, key, patches, module, lora_mode):
        self.key, self.patches, self.module, self.lora_mode = key, patches, module, lora_mode
        self.prepared_patches = None

    def memory_required(self):
        return 0

    def prepare(self, *args, **kwargs):
        self.prepared_patches = list(self.patches[self.key])
        return self.prepared_patches

    def clear_prepared(self):
        self.prepared_patches = None

    def _current_patches(self):
        return self.patches[self.key] if self.prepared_patches is None else self.prepared_patches

    def __call__(self, weight):
        return self.apply(weight, self._current_patches())

    def apply(self, weight, patches):
        raise NotImplementedError
