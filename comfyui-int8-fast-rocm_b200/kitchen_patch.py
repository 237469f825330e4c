"""comfy_kitchen ``int8_linear`` override backed by the sm_100a kernels
(reference: rocm_int8_kitchen_patch.py).

``int8_linear`` keeps the kitchen op's signature and behaviour
(rocm_int8_kitchen_patch.py:114-176): SiTU / kitchen input activation,
shape and scale validation with the same ValueErrors, optional ConvRot
(fused into the quantisation kernel here), the W8A8 GEMM with per-tensor or
per-channel weight scale, and kitchen's residual form.  The RMS-norm input
activation (``dt((x * rsqrt(mean(x^2) + eps)) * weight)``, F.rms_norm's
rounding) runs inside the activation quantiser, and ``residual +
residual_scale * y`` inside the GEMM epilogue, whenever the dtypes keep the
eager result in the output dtype; other cases take kitchen's own helpers.  ``apply_patch``
installs it in kitchen's registry and in the modules that import
``int8_linear`` directly; it runs on import when comfy_kitchen is present.
The reference's ROCm architecture gating is not carried over (this build is
sm_100a-only).
"""
from __future__ import annotations

import logging

import torch

from . import library as kops  # the kernels as registered torch.library operators
from .int8_quant import rot_for_group

log = logging.getLogger("comfyui-int8-fast-b200")

try:
    import comfy_kitchen.backends.eager.quantization as ck_quant
    from comfy_kitchen.registry import registry
except ImportError:  # kitchen absent: the function is still usable directly
    ck_quant = None
    registry = None

try:
    import comfy_kitchen.backends.eager.w4a8_int8 as ck_w4a8_eager
except ImportError:
    ck_w4a8_eager = None


RMS_INPUT_ACTS = ("rms_norm", "rmsnorm")


def _fusable_rms(x, input_act, input_act_weight) -> bool:
    """The RMS-norm input activation runs inside the quantiser for 16-bit
    rows of 16-element multiples (with a [K] weight or none)."""
    return (input_act in RMS_INPUT_ACTS and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)
            and x.shape[-1] % 16 == 0
            and (input_act_weight is None or input_act_weight.numel() == x.shape[-1]))


def _fusable_residual(residual, residual_scale, out_shape, out_dtype) -> bool:
    """``residual + residual_scale * y`` runs in the GEMM epilogue when the
    result keeps ``out_dtype`` (residual of that dtype and of the output's
    shape; scale absent or one ``out_dtype`` value per output feature)."""
    if residual is None or out_dtype not in (torch.bfloat16, torch.float16) or out_shape[-1] % 8:
        return False
    if residual.dtype != out_dtype or tuple(residual.shape) != tuple(out_shape):
        return False
    if residual_scale is None:
        return True
    return (isinstance(residual_scale, torch.Tensor) and residual_scale.dtype == out_dtype
            and residual_scale.numel() == out_shape[-1] and residual_scale.shape[-1] == out_shape[-1])


def int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias=None,
                out_dtype: torch.dtype = torch.bfloat16, convrot: bool = False, convrot_groupsize: int = 256,
                input_act=None, input_act_weight=None, input_act_eps: float = 0.0, residual=None,
                residual_scale=None) -> torch.Tensor:
    # SiTU of 16-bit rows of 16-element multiples runs inside the activation
    # quantiser (bit-equal to kops.situ followed by kops.quant_act_int8)
    fuse_situ = (input_act == "situ" and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)
                 and x.shape[-1] % 32 == 0)
    if input_act == "situ" and not fuse_situ:
        x = kops.situ(x)
    if input_act == "situ":
        input_act = None
    k_in = x.shape[-1] // 2 if fuse_situ else x.shape[-1]
    fuse_rms = _fusable_rms(x, input_act, input_act_weight)
    if fuse_rms or fuse_situ:
        pass  # applied inside the activation quantiser below
    elif ck_quant is not None:
        x = ck_quant._apply_input_act(x, input_act, input_act_weight, input_act_eps)
    elif input_act is not None:
        raise ValueError(f"input_act={input_act!r} needs comfy_kitchen")
    if k_in != weight.shape[-1]:
        raise ValueError(f"Input and weight inner dimensions must match, got {k_in} and {weight.shape[-1]}")
    weight = weight.to(device=x.device).contiguous()
    weight_scale = weight_scale.to(device=x.device, dtype=torch.float32).reshape(-1)
    if weight_scale.numel() not in (1, weight.shape[0]):
        raise ValueError(f"INT8 weight scale must be scalar or per-output-channel, got {tuple(weight_scale.shape)} "
                         f"for weight shape {tuple(weight.shape)}")
    rot = None
    if convrot:
        if k_in % convrot_groupsize != 0:
            raise ValueError(f"ConvRot group size {convrot_groupsize} does not divide input features {k_in}")
        rot = rot_for_group(convrot_groupsize)
    shape = (*x.shape[:-1], k_in)
    x2 = x.reshape(-1, x.shape[-1])
    if fuse_situ:
        xq, xs = kops.quant_act_int8_situ(x2, rot)
    elif fuse_rms:
        xq, xs = kops.quant_act_int8_norm(x2, rot, "rms", float(input_act_eps), input_act_weight)
    else:
        xq, xs = kops.quant_act_int8(x2, rot)
    out_shape = (*shape[:-1], weight.shape[0])
    per_row = weight_scale.numel() > 1
    if _fusable_residual(residual, residual_scale, out_shape, out_dtype):
        out = kops.gemm_w8a8_fused(xq, xs, weight, weight_scale, bias, out_dtype, per_row=per_row,
                                  residual=residual.reshape(-1, weight.shape[0]),
                                  gate=None if residual_scale is None else residual_scale.reshape(1, -1))
        return out.reshape(out_shape)
    out = kops.gemm_w8a8(xq, xs, weight, weight_scale, bias, out_dtype, per_row=per_row)
    out = out.reshape(out_shape)
    if ck_quant is not None:
        return ck_quant._apply_residual(out, residual, residual_scale)
    if residual is not None:
        out = residual + (out if residual_scale is None else residual_scale * out)
    return out


_original_get_implementation = getattr(registry, "get_implementation", None)


def _patched_get_implementation(name, *args, **kwargs):
    if name == "int8_linear":
        return int8_linear
    return _original_get_implementation(name, *args, **kwargs)


def apply_patch() -> bool:
    """Route kitchen's ``int8_linear`` to this build (registry lookup and
    the modules that bound the function at import time)."""
    if registry is None:
        return False
    registry.get_implementation = _patched_get_implementation
    ck_quant.int8_linear = int8_linear
    if ck_w4a8_eager is not None:
        ck_w4a8_eager.int8_linear = int8_linear
    log.info("comfy_kitchen int8_linear -> sm_100a kernels")
    return True


apply_patch()
