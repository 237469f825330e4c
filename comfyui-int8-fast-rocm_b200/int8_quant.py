"""W8A8 quantisation math and the ``Int8TensorwiseOps`` ComfyUI custom
operations (reference: int8_quant.py).

Module-level functions keep the reference's names and semantics
(int8_quant.py:41-164) but run on the sm_100a kernels; they take CUDA
tensors.  ``Int8TensorwiseOps`` is defined when ComfyUI's ``comfy.ops`` is
importable, with the same class-level flags, state-dict formats and forward
contract as the reference (int8_quant.py:170-747); its forward is one fused
rotate+quantise launch plus one tcgen05 GEMM launch.
"""
from __future__ import annotations

import json
import logging

import torch
from torch import Tensor, nn
import torch.nn.functional as F

from . import library as kops  # the kernels as registered torch.library operators
from .linear_common import (QuantLowVramPatch, calc_weight_entries, float_forward, init_linear, scale_layout,
                            store_param)

# Runtime toggle kept for API compatibility (the reference switches between
# Triton and torch._int_mm with it); this build always runs its own kernels.
_use_triton = True

# ConvRot group size used for on-the-fly quantisation (int8_quant.py:37)
CONVROT_GROUP_SIZE = 256


def rot_for_group(group_size: int):
    """(kind, group) for a ConvRot group size: the reference's regular
    construction for powers of 4, Sylvester otherwise (e.g. 128)."""
    g = int(group_size)
    kind = "regular" if (g & (g - 1)) == 0 and (g.bit_length() - 1) % 2 == 0 else "sylvester"
    return kind, g


# --- Quantisation utils (int8_quant.py:41-55) --------------------------------


def _rows2d(x: Tensor) -> Tensor:
    return x.reshape(-1, x.shape[-1])


def quantize_int8(x: Tensor, scale) -> Tensor:
    """round(x.float() * (1/scale)).clamp(-128, 127) -> int8 with a given
    scalar or per-row [N,1] scale."""
    return kops.requant_int8(_rows2d(x.float()), scale).reshape(x.shape)


def quantize_int8_tensorwise(x: Tensor):
    """(q, scale) with one absmax/127 scale for the whole tensor."""
    scale = (x.abs().max().float() / 127.0).clamp(min=1e-30)
    return quantize_int8(x, scale), scale


def quantize_int8_axiswise(x: Tensor, dim: int):
    """Per-axis absmax int8 along the last axis (dim=-1 for activations,
    dim=1 for a 2-D weight)."""
    if dim not in (-1, x.dim() - 1):
        raise ValueError("quantize_int8_axiswise supports the last axis (dim=-1, or dim=1 for 2-D weights)")
    q, s = kops.quant_act_int8(_rows2d(x))
    return q.reshape(x.shape), s.reshape(tuple(x.shape[:-1]) + (1,))


def dequantize(q: Tensor, scale) -> Tensor:
    """q.float() * scale (float32)."""
    return kops.dequant_int8(_rows2d(q), scale).reshape(q.shape)


def stochastic_round_int8_delta(x: Tensor, scale, seed: int = 0) -> Tensor:
    """Stochastic int8 rounding of x/scale (int8_quant.py:80-106): floor +1
    with probability equal to the fraction.  The kernel's counter-based RNG
    draws differ from torch.Generator's stream (same law)."""
    return kops.requant_int8(_rows2d(x.float()), scale, stochastic=True, seed=seed).reshape(x.shape)


# --- W8A8 forward (int8_quant.py:113-164) ------------------------------------


@torch.no_grad()
def int8_forward_dynamic(x: Tensor, weight: Tensor, weight_scale, bias, compute_dtype, rot=None) -> Tensor:
    """Per-token activation quant + W8A8 GEMM with a scalar weight scale."""
    xq, xs = kops.quant_act_int8(x, rot)
    if not isinstance(weight_scale, torch.Tensor):
        weight_scale = torch.tensor([float(weight_scale)], dtype=torch.float32, device=x.device)
    return kops.gemm_w8a8(xq, xs, weight, weight_scale, bias, compute_dtype, per_row=False)


@torch.no_grad()
def int8_forward_dynamic_per_row(x: Tensor, weight: Tensor, weight_scale: Tensor, bias, compute_dtype,
                                 rot=None) -> Tensor:
    """Per-token activation quant + W8A8 GEMM with per-row weight scales."""
    xq, xs = kops.quant_act_int8(x, rot)
    return kops.gemm_w8a8(xq, xs, weight, weight_scale, bias, compute_dtype, per_row=True)


@torch.no_grad()
def int8_forward_fused(x: Tensor, weight: Tensor, weight_scale, bias, compute_dtype, rot=None, per_row=True, *,
                       norm=None, eps: float = 1e-6, norm_weight=None, mod_mul=None, mod_add=None,
                       rows_per_sample=None, gelu_from=None, residual=None, gate=None,
                       rows_per_gate=None, x2=None, out=None, out_rows=None) -> Tensor:
    """:func:`int8_forward_dynamic_per_row` / :func:`int8_forward_dynamic`
    with the element-wise neighbours of a DiT block's linear fused into its
    two kernels (no counterpart in the reference, which runs them as eager
    ops around ``Int8TensorwiseOps.Linear``):

    * prologue (activation quantiser): ``dt(norm(x))`` (``norm`` "layer" or
      "rms" with ``norm_weight``), ``dt(. * mod_mul[s])``, ``dt(. +
      mod_add[s])`` with ``s = row // rows_per_sample`` -- a Flux block's
      ``layer_norm(x) * (1 + scale) + shift`` is ``norm="layer",
      mod_mul=1 + scale, mod_add=shift``;
    * epilogue (GEMM): ``dt(gelu_tanh(y))`` on columns ``>= gelu_from``, then
      ``dt(residual + dt(gate[g] * y))`` with ``g = row // rows_per_gate``;
    * ``x2``: the linear's input is ``torch.cat((x, x2), -1)``, read from the
      two tensors by the quantiser (no prologue steps then);
    * ``out_rows=(n, stride, off)``: output row r lands in row
      ``(r // n) * stride + off + r % n`` of ``out`` (see
      ``ops.gemm_w8a8_fused``), e.g. one stream's q/k/v rows written straight
      into the joint sequence of a double block.
    """
    prologue = norm is not None or mod_mul is not None or mod_add is not None
    if x2 is not None:
        if prologue:
            raise ValueError("a concatenated input takes no norm / modulation prologue")
        xq, xs = kops.quant_act_int8_cat(x, x2, rot)
    elif prologue:
        xq, xs = kops.quant_act_int8_norm(x, rot, norm, eps, norm_weight, mod_mul, mod_add, rows_per_sample)
    else:
        xq, xs = kops.quant_act_int8(x, rot)
    if not per_row and not isinstance(weight_scale, torch.Tensor):
        weight_scale = torch.tensor([float(weight_scale)], dtype=torch.float32, device=x.device)
    if gelu_from is None and residual is None and out is None:
        return kops.gemm_w8a8(xq, xs, weight, weight_scale, bias, compute_dtype, per_row=per_row)
    return kops.gemm_w8a8_fused(xq, xs, weight, weight_scale, bias, compute_dtype, per_row=per_row,
                               gelu_from=gelu_from, residual=residual, gate=gate, rows_per_gate=rows_per_gate,
                               out=out, out_rows=out_rows)


def lowvram_patch_int8(weight: Tensor, scale, convrot_groupsize, delta_fn, stochastic=False, seed=0) -> Tensor:
    """INT8LowVramPatch.__call__ / bake-in path (int8_quant.py:809-843,
    881-941) on the kernels: dequant (+ un-rotate) -> ``delta_fn`` (the
    float-space patch, e.g. comfy.lora.calculate_weight) -> re-rotate ->
    requantise with the ORIGINAL scale (RNE or stochastic)."""
    rot = rot_for_group(convrot_groupsize) if convrot_groupsize else None
    w = kops.dequant_int8(weight, scale, rot)
    w = delta_fn(w)
    return kops.requant_int8(w, scale, rot, stochastic=stochastic, seed=seed)


# =============================================================================
# Int8TensorwiseOps -- ComfyUI custom operations
# =============================================================================

try:
    from comfy.ops import manual_cast, cast_bias_weight, uncast_bias_weight
    _COMFY_OPS_AVAILABLE = True
except ImportError:
    _COMFY_OPS_AVAILABLE = False


def _parse_comfy_quant(t):
    if t is None:
        return None
    try:
        return json.loads(bytes(t.tolist()).decode("utf-8"))
    except Exception:
        return None


def _pop_metadata(sd, p, k):
    """Tolerate 'model.' / 'diffusion_model.' prefixes (int8_quant.py:369-380)."""
    v = sd.pop(p + k, None)
    if v is not None:
        return v
    v = sd.pop("model." + p + k, None)
    if v is not None:
        return v
    if p.startswith("model."):
        v = sd.pop(p[6:] + k, None)
        if v is not None:
            return v
    if p.startswith("diffusion_model."):
        v = sd.pop("diffusion_model." + p + k, None)
        if v is not None:
            return v
    return None


def _normalize_lora_key(key):
    if not isinstance(key, str):
        return key
    for p in ["diffusion_model.", "model.diffusion_model.", "model.", "transformer."]:
        if key.startswith(p):
            return key[len(p):]
    return key


if _COMFY_OPS_AVAILABLE:

    class Int8TensorwiseOps(manual_cast):
        """ComfyUI custom operations for INT8 W8A8 linears (int8_quant.py:170-747)."""

        excluded_names = []
        dynamic_quantize = False
        enable_convrot = False
        use_triton = True
        compute_dtype = None
        _is_prequantized = False
        lora_mode = "None"
        dynamic_lora = False
        lora_patches = {}
        lora_strength = 1.0
        dynamic_load_device = None
        skeleton_meta_init = False
        _auto_compute_dtype_by_device = {}

        @staticmethod
        def _default_compute_dtype(x: Tensor) -> torch.dtype:
            if x.dtype in (torch.float16, torch.bfloat16):
                return x.dtype
            return torch.float16

        class Linear(manual_cast.Linear):
            def __init__(self, in_features, out_features, bias=True, device=None, dtype=None):
                init_linear(self, Int8TensorwiseOps, super().__init__, in_features, out_features, bias, device, dtype)
                self.register_buffer("weight_scale", None)
                self._is_quantized = False
                self._is_per_row = False
                self._use_convrot = False
                self._convrot_groupsize = CONVROT_GROUP_SIZE
                self._weight_scale_scalar = None
                self.compute_dtype = None
                self.comfy_cast_weights = False
                self.lora_patches = []
                self._w4a8_cache = {}

            def reset_parameters(self):
                return None

            _normalize_lora_key = staticmethod(_normalize_lora_key)

            @staticmethod
            def _is_bias_key(key):
                return isinstance(key, str) and key.endswith(".bias")

            @staticmethod
            def _format_lora_patches(patches):
                """Grouped pre-LoRA entries as comfy.lora.calculate_weight
                entries (int8_quant.py:256-265)."""
                return calc_weight_entries(patches, getattr(Int8TensorwiseOps, "lora_strength", 1.0))

            def _apply_int8_lora_patches(self, tensor, key, patches, device):
                """Bake pre-LoRA patches into a float weight in ComfyUI's LoRA
                compute dtype (int8_quant.py:268-274)."""
                if not patches or tensor.dtype == torch.int8:
                    return tensor
                import comfy.lora
                import comfy.model_management
                temp_dtype = comfy.model_management.lora_compute_dtype(device)
                tensor_temp = tensor.to(device, non_blocking=True).to(dtype=temp_dtype)
                return comfy.lora.calculate_weight(self._format_lora_patches(patches), tensor_temp, key)

            def finalize_pending_int8(self):
                """Deferred load work (pre-LoRA bake and/or on-the-fly quant)
                recorded while a dynamic load device was set; run by
                INT8ModelPatcher at model load (int8_quant.py:276-325)."""
                pending = getattr(self, "_pending_int8_finalize", None)
                if pending is None:
                    return False
                device = pending.get("device") or torch.device("cuda")
                weight_tensor = self._apply_int8_lora_patches(
                    self.weight.detach(), pending["weight_key"], pending.get("lora_patches"), device)
                if pending["quantize"]:
                    saved = Int8TensorwiseOps.enable_convrot
                    Int8TensorwiseOps.enable_convrot = pending.get("enable_convrot", False)
                    try:
                        self._otf_quantize(weight_tensor.to(device))
                    finally:
                        Int8TensorwiseOps.enable_convrot = saved
                else:
                    self.weight = nn.Parameter(weight_tensor.cpu(), requires_grad=False)
                self.weight_comfy_model_dtype = self.weight.dtype
                if self.weight_scale is not None:
                    self.weight_scale_comfy_model_dtype = self.weight_scale.dtype
                if self.bias is not None:
                    self.bias_comfy_model_dtype = self.bias.dtype
                del self._pending_int8_finalize
                return True

            # -- loading ----------------------------------------------------
            def _otf_quantize(self, weight_tensor):
                """On-the-fly quant (int8_quant.py:517-554): float32 weight ->
                optional ConvRot -> per-row int8, kept on the CPU like the
                reference (moved per forward or by the model patcher)."""
                device = getattr(Int8TensorwiseOps, "dynamic_load_device", None) or torch.device("cuda")
                w = weight_tensor.to(device, non_blocking=True)
                self._use_convrot = False
                rot = None
                if getattr(Int8TensorwiseOps, "enable_convrot", False) and self.in_features % CONVROT_GROUP_SIZE == 0:
                    rot = rot_for_group(CONVROT_GROUP_SIZE)
                    self._use_convrot = True
                    self._convrot_groupsize = CONVROT_GROUP_SIZE
                q, s = kops.quant_weight_int8(w, rot)
                self.weight = nn.Parameter(q.cpu(), requires_grad=False)
                self.register_buffer("weight_scale", s.cpu())
                self._weight_scale_scalar = None
                self._is_quantized = True
                self._is_per_row = True

            # pre-LoRA patches grouped by the loader (int8_quant.py:335-453) are
            # baked into float weights and biases before any quantisation, or
            # deferred to model load when a dynamic load device is set
            @staticmethod
            def _pre_lora_patches(key):
                table = Int8TensorwiseOps.lora_patches
                return table.get(_normalize_lora_key(key)) if table else None

            @staticmethod
            def _mark_pre_lora_applied(key):
                if getattr(Int8TensorwiseOps, "applied_lora_patches", None) is None:
                    Int8TensorwiseOps.applied_lora_patches = set()
                Int8TensorwiseOps.applied_lora_patches.add(_normalize_lora_key(key))

            def _bake_pre_lora(self, tensor, key):
                if tensor is None or tensor.dtype == torch.int8:
                    return tensor
                patches = self._pre_lora_patches(key)
                if not patches:
                    return tensor
                self._mark_pre_lora_applied(key)
                device = getattr(Int8TensorwiseOps, "dynamic_load_device", None) or tensor.device
                return self._apply_int8_lora_patches(tensor, key, patches, device).to(tensor.dtype)

            def _keep_float(self, weight):
                self._is_quantized = False
                self.weight = nn.Parameter(weight, requires_grad=False)

            def _set_quantized_weight(self, weight, per_row):
                self.weight = nn.Parameter(weight, requires_grad=False)
                self._is_quantized = True
                self._is_per_row = per_row
                Int8TensorwiseOps._is_prequantized = True

            def _take_asym_w4a8(self, state_dict, prefix, weight, conf, wkey):
                """asym_w4a8_int8 layer (w4a8_int8.py layout): packed codes
                plus codebook, channel and group scales; False (and the layer
                falls through to the generic path) when a part is missing."""
                if weight is None or weight.dtype != torch.int8:
                    logging.warning(f"asym W4A8: no packed int8 codes under {wkey}; loading the layer as stored")
                    return False
                parts = [_pop_metadata(state_dict, prefix, f"weight_{n}") for n in ("codebook", "s_channel", "s_rel")]
                if any(t is None for t in parts):
                    logging.warning(f"asym W4A8: {wkey} comes without codebook or scales; loading the layer as stored")
                    return False
                self._w4a8_codebook, self._w4a8_s_channel, self._w4a8_s_rel = parts
                self._w4a8_group_size = int(conf.get("group_size", 16))
                self._is_w4a8 = True
                self._set_quantized_weight(weight, per_row=True)
                return True

            def _take_float(self, weight, prefix, wkey, pending_lora):
                """A float weight: quantised now (on the fly), at model load
                (dynamic load device), or kept in its precision (excluded
                layers, vectors, quantisation off)."""
                ops = Int8TensorwiseOps
                quantize = (ops.dynamic_quantize and not any(ex in prefix for ex in ops.excluded_names)
                            and 1 not in (self.in_features, self.out_features) and weight.ndim != 1)
                load_dev = getattr(ops, "dynamic_load_device", None)
                if load_dev is not None and (quantize or pending_lora):
                    self._keep_float(weight)
                    self._pending_int8_finalize = {"weight_key": wkey, "quantize": quantize, "lora_patches": pending_lora,
                                                   "device": load_dev,
                                                   "enable_convrot": getattr(ops, "enable_convrot", False)}
                    if pending_lora:
                        self._mark_pre_lora_applied(wkey)
                elif quantize:
                    if not getattr(ops, "_logged_otf", False):
                        logging.info(f"INT8 Fast B200: on-the-fly W8A8 quantisation while loading "
                                     f"(ConvRot {'on' if ops.enable_convrot else 'off'})")
                        ops._logged_otf = True
                    self._otf_quantize(weight)
                else:
                    self._keep_float(weight)

            def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs):
                """The layer's tensors in any of the formats of
                int8_quant.py:328-577: asym_w4a8_int8, int8 with a
                weight_scale (per row or tensor-wide, optional ConvRot), or a
                float weight."""
                wkey, bkey = prefix + "weight", prefix + "bias"
                scale = _pop_metadata(state_dict, prefix, "weight_scale")
                conf = _parse_comfy_quant(_pop_metadata(state_dict, prefix, "comfy_quant"))
                conf = conf if isinstance(conf, dict) else {}
                weight, bias = state_dict.pop(wkey, None), state_dict.pop(bkey, None)
                state_dict.pop(prefix + "input_scale", None)

                pending_lora = (self._pre_lora_patches(wkey)
                                if weight is not None and weight.dtype != torch.int8 else None)
                if not (pending_lora and getattr(Int8TensorwiseOps, "dynamic_load_device", None) is not None):
                    weight = self._bake_pre_lora(weight, wkey)
                bias = self._bake_pre_lora(bias, bkey)
                if conf.get("convrot", False):
                    self._use_convrot = True
                    Int8TensorwiseOps.enable_convrot = True
                    self._convrot_groupsize = int(conf.get("convrot_groupsize", self._convrot_groupsize))

                if conf.get("format") == "asym_w4a8_int8" and self._take_asym_w4a8(state_dict, prefix, weight, conf,
                                                                                   wkey):
                    pass
                elif weight is None:
                    missing_keys.append(wkey)
                elif weight.dtype == torch.int8 and scale is not None:
                    buf, per_row = scale_layout(scale, conf.get("per_row"))
                    self._set_quantized_weight(weight, per_row)
                    self.register_buffer("weight_scale", buf)
                elif weight.dtype in (torch.float16, torch.bfloat16, torch.float32):
                    self._take_float(weight, prefix, wkey, pending_lora)
                else:
                    self._keep_float(weight)

                self.bias = nn.Parameter(bias, requires_grad=False) if bias is not None else None
                for name in ("weight", "weight_scale", "bias"):
                    t = getattr(self, name)
                    if t is not None:
                        setattr(self, f"{name}_comfy_model_dtype", t.dtype)

            def _get_weight_scale(self):
                return self.weight_scale

            def convert_weight(self, _weight, inplace=False):
                if not self._is_quantized:
                    return _weight
                return self.weight

            def set_weight(self, out_weight, inplace_update=False, seed=0, return_weight=False, **kwargs):
                if not self._is_quantized:
                    value = out_weight.to(self.weight.dtype)
                elif out_weight.dtype == torch.int8:
                    value = out_weight
                else:  # a float patch result: requantised with the layer's own scale
                    value = quantize_int8(out_weight, self._get_weight_scale().to(out_weight.device))
                return store_param(self, "weight", value, inplace_update, return_weight)

            def set_bias(self, out_bias, inplace_update=False, seed=0, return_weight=False, **kwargs):
                if out_bias is None:
                    return None
                return store_param(self, "bias", out_bias, inplace_update, return_weight)

            # -- forward ----------------------------------------------------
            def _w4a8_int8_weight(self, weight):
                """asym_w4a8_int8 -> per-channel int8, computed once per device
                by the fused dequant+requant kernel and cached (the reference
                recomputes it every call, int8_quant.py:679-687)."""
                key = (weight.device, weight.data_ptr())
                hit = self._w4a8_cache.get(key)
                if hit is None:
                    hit = kops.requant_asym_w4a8(weight, self._w4a8_codebook, self._w4a8_s_channel,
                                                self._w4a8_s_rel, self._w4a8_group_size)
                    self._w4a8_cache = {key: hit}
                return hit

            def forward(self, x: Tensor) -> Tensor:
                need_cast = self.comfy_cast_weights or len(self.weight_function) > 0 or len(self.bias_function) > 0
                if not self._is_quantized:
                    return float_forward(self, x, need_cast, cast_bias_weight, uncast_bias_weight)

                if need_cast:
                    weight, bias, offload_stream = cast_bias_weight(
                        self, input=None, dtype=torch.int8, device=x.device, bias_dtype=x.dtype, offloadable=True)
                else:
                    weight, bias, offload_stream = self.weight, self.bias, None
                if weight is not None and weight.device != x.device:
                    weight = weight.to(x.device, non_blocking=True)
                if bias is not None and bias.device != x.device:
                    bias = bias.to(x.device, non_blocking=True)

                if getattr(self, "_is_w4a8", False):
                    weight, w_scale = self._w4a8_int8_weight(weight)
                else:
                    w_scale = self._get_weight_scale()
                    if isinstance(w_scale, torch.Tensor) and w_scale.device != x.device:
                        w_scale = w_scale.to(x.device, non_blocking=True)

                compute_dtype = Int8TensorwiseOps.compute_dtype or Int8TensorwiseOps._default_compute_dtype(x)
                x_shape = x.shape
                x_2d = x.reshape(-1, x_shape[-1])
                if x_2d.dtype != compute_dtype:
                    x_2d = x_2d.to(compute_dtype)
                rot = rot_for_group(self._convrot_groupsize) if self._use_convrot else None

                patches = self.lora_patches
                if (len(patches) == 1 and patches[0][2] is None
                        and compute_dtype in (torch.bfloat16, torch.float16)):
                    # one full-width dynamic LoRA: y + lora_y.to(y.dtype) is the
                    # GEMM epilogue's residual step (dt(y + residual), one
                    # rounding at the store), so the sum is bit-equal to the
                    # eager add and y is written once
                    lora_down, lora_up = patches[0][0], patches[0][1]
                    x_l = kops.rotate(x_2d, *rot) if rot is not None else x_2d
                    lD = lora_down.to(x.device, non_blocking=True)
                    lU = lora_up.to(x.device, non_blocking=True)
                    lora_y = F.linear(F.linear(x_l.to(lD.dtype), lD), lU).to(compute_dtype)
                    y = int8_forward_fused(x_2d, weight, w_scale, bias, compute_dtype, rot,
                                           per_row=self._is_per_row, residual=lora_y)
                    patches = []
                elif self._is_per_row:
                    y = int8_forward_dynamic_per_row(x_2d, weight, w_scale, bias, compute_dtype, rot)
                else:
                    y = int8_forward_dynamic(x_2d, weight, w_scale, bias, compute_dtype, rot)

                if patches:
                    # dynamic LoRA (int8_quant.py:718-729): down-projection of
                    # the (rotated) activation, up-projection, added to y
                    x_l = kops.rotate(x_2d, *rot) if rot is not None else x_2d
                    for lora_down, lora_up, lora_start, lora_size in patches:
                        lD = lora_down.to(x.device, non_blocking=True)
                        lU = lora_up.to(x.device, non_blocking=True)
                        lora_y = F.linear(F.linear(x_l.to(lD.dtype), lD), lU)
                        if lora_start is not None:
                            y[:, lora_start:lora_start + lora_size] = (
                                y[:, lora_start:lora_start + lora_size] + lora_y.to(y.dtype))
                        else:
                            y = y + lora_y.to(y.dtype)

                if need_cast:
                    uncast_bias_weight(self, weight, bias, offload_stream)
                return y.reshape(*x_shape[:-1], y.shape[-1])

        class GroupNorm(manual_cast.GroupNorm):
            pass

        class LayerNorm(manual_cast.LayerNorm):
            pass

        class Conv2d(manual_cast.Conv2d):
            pass

        class Conv3d(manual_cast.Conv3d):
            pass

        class ConvTranspose2d(manual_cast.ConvTranspose2d):
            pass

        class Embedding(manual_cast.Embedding):
            pass

        @classmethod
        def conv_nd(cls, dims, *args, **kwargs):
            if dims == 2:
                return cls.Conv2d(*args, **kwargs)
            if dims == 3:
                return cls.Conv3d(*args, **kwargs)
            raise ValueError(f"unsupported dimensions: {dims}")


# =============================================================================
# LoRA on INT8 layers: low-VRAM patch callable and the model patcher
# =============================================================================

try:
    import comfy.model_patcher as _comfy_model_patcher
    import comfy.lora as _comfy_lora
    import comfy.utils as _comfy_utils
    _COMFY_PATCHER_AVAILABLE = _COMFY_OPS_AVAILABLE
except ImportError:
    _COMFY_PATCHER_AVAILABLE = False


def _int8_module_rot(module):
    """The (kind, group) rotation of an INT8 layer, or None."""
    if getattr(module, "_use_convrot", False):
        return rot_for_group(getattr(module, "_convrot_groupsize", CONVROT_GROUP_SIZE))
    return None


def _dynamic_lora_entries(module, patches, rot, group_ok):
    """Dynamic-LoRA (down_scaled, up, start, size) entries for one layer
    (int8_quant.py:969-1008): the LoRA down projection is scaled by
    alpha/rank * strength and, for a ConvRot layer, rotated like the weight
    (W_rot = W H^T  =>  dW_rot = up (down H^T))."""
    entries = []
    for p in patches:
        strength_patch, adapter, strength_model = p[0], p[1], p[2]
        offset = p[3] if len(p) > 3 else None
        if not hasattr(adapter, "weights"):
            continue
        weights = adapter.weights
        if len(weights) != 6:
            continue
        up, down, alpha, mid, _dora, _reshape = weights
        strength = strength_patch * strength_model
        rank = down.shape[0] if down.ndim >= 2 else 1
        scale = (alpha / rank) * strength if alpha is not None else strength
        down_scaled = down.flatten(1) * scale
        if mid is not None:
            down_scaled = torch.mm(mid.flatten(1), down.flatten(1)) * scale
        if rot is not None and group_ok(down_scaled.shape[1]):
            down_scaled = kops.rotate(down_scaled.to(torch.float32).cuda(), *rot).to(down_scaled.dtype)
        start = size = None
        if offset is not None:
            _dim, start, size = offset
        entries.append((down_scaled, up.flatten(1), start, size))
    return entries


if _COMFY_PATCHER_AVAILABLE:

    class INT8LowVramPatch(QuantLowVramPatch):
        """Low-VRAM LoRA on an INT8 layer as ComfyUI streams the weight in
        (int8_quant.py:761-843): dequant (+ un-rotate) -> patch in float ->
        re-rotate -> requantise with the layer's original scale."""

        def apply(self, weight, patches):
            scale = self.module._get_weight_scale()
            if isinstance(scale, torch.Tensor):
                scale = scale.to(weight.device)
            rot = _int8_module_rot(self.module)
            stochastic = self.lora_mode == "Stochastic"
            return lowvram_patch_int8(
                weight, scale, rot[1] if rot else 0,
                lambda w: _comfy_lora.calculate_weight(patches, w, self.key, intermediate_dtype=w.dtype),
                stochastic=stochastic, seed=_comfy_utils.string_to_seed(self.key) if stochastic else 0)

    class INT8ModelPatcher(_comfy_model_patcher.ModelPatcher):
        """ModelPatcher that routes LoRA patches on INT8 layers through the
        bake-in path (dequant -> patch -> requant, on the kernels) or the
        dynamic path (low-rank branch in the forward), per
        ``Int8TensorwiseOps.dynamic_lora`` (int8_quant.py:846-1110)."""

        def finalize_pending_int8(self):
            finalized = 0
            for module in self.model.modules():
                fn = getattr(module, "finalize_pending_int8", None)
                if fn is not None and fn():
                    finalized += 1
            if finalized:
                self.size = 0
                torch.cuda.empty_cache()
            return finalized

        def _int8_module(self, key):
            try:
                module = _comfy_utils.get_attr(self.model, key.rsplit(".", 1)[0])
            except AttributeError:
                return None
            return module if getattr(module, "_is_quantized", False) else None

        def patch_weight_to_device(self, key, device_to=None, inplace_update=False, return_weight=False,
                                   force_cast=False):
            if key not in self.patches and not force_cast:
                return super().patch_weight_to_device(key, device_to, inplace_update, return_weight, force_cast)
            module = self._int8_module(key)
            if module is None:
                return super().patch_weight_to_device(key, device_to, inplace_update, return_weight, force_cast)
            if Int8TensorwiseOps.Linear._is_bias_key(key):
                return _comfy_utils.get_attr(self.model, key) if return_weight else None
            patches = self.patches.get(key, [])

            if not Int8TensorwiseOps.dynamic_lora:
                # bake: always from the backed-up base weight (no stacking)
                current = _comfy_utils.get_attr(self.model, key)
                if device_to is None:
                    device_to = current.device
                if key not in self.backup:
                    import collections
                    Backup = collections.namedtuple("Dimension", ["weight", "inplace_update"])
                    self.backup[key] = Backup(weight=current.to(device=self.offload_device, copy=inplace_update),
                                              inplace_update=inplace_update)
                    source = current
                else:
                    source = self.backup[key].weight
                dev = device_to if torch.device(device_to).type == "cuda" else torch.device("cuda")
                scale = module._get_weight_scale()
                if isinstance(scale, torch.Tensor):
                    scale = scale.to(dev)
                group = getattr(module, "_convrot_groupsize", CONVROT_GROUP_SIZE) \
                    if getattr(module, "_use_convrot", False) else 0
                stochastic = getattr(Int8TensorwiseOps, "lora_mode", "None") == "Stochastic"
                patched = lowvram_patch_int8(
                    source.to(dev), scale, group,
                    lambda w: _comfy_lora.calculate_weight(patches, w, key),
                    stochastic=stochastic, seed=_comfy_utils.string_to_seed(key) if stochastic else 0)
                patched = patched.to(current.device)
                if return_weight:
                    return patched
                if inplace_update:
                    current.data.copy_(patched)
                else:
                    _comfy_utils.set_attr(self.model, key, nn.Parameter(patched, requires_grad=False))
                return None

            # dynamic: low-rank branch evaluated in Linear.forward
            weight = _comfy_utils.get_attr(self.model, key)
            cache_key = tuple(id(p[1]) for p in patches)
            if getattr(module, "_lora_cache_key", None) != cache_key:
                device = weight.device if weight is not None else self.offload_device
                rot = _int8_module_rot(module)
                entries = _dynamic_lora_entries(module, patches, rot, lambda k: k % rot[1] == 0 if rot else False)
                module.lora_patches = [(d.to(device), u.to(device), s0, sz) for d, u, s0, sz in entries]
                module._lora_cache_key = cache_key
            return weight if return_weight else None

        def load(self, *args, **kwargs):
            self.finalize_pending_int8()
            if not Int8TensorwiseOps.dynamic_lora:
                # restore the base INT8 weights so the bake starts from them
                for k in list(self.backup):
                    if k in self.patches and self._int8_module(k) is not None:
                        bk = self.backup.pop(k)
                        if bk.inplace_update:
                            _comfy_utils.get_attr(self.model, k).data.copy_(bk.weight)
                        else:
                            _comfy_utils.set_attr(self.model, k, bk.weight)
            for k in [k for k in self.backup if k not in self.patches]:  # stale patches
                bk = self.backup.pop(k)
                if bk.inplace_update:
                    _comfy_utils.get_attr(self.model, k).data.copy_(bk.weight)
                else:
                    _comfy_utils.set_attr(self.model, k, bk.weight)
            for name, module in self.model.named_modules():
                if getattr(module, "lora_patches", None):
                    if not Int8TensorwiseOps.dynamic_lora or (name + ".weight") not in self.patches:
                        module.lora_patches = []
            res = super().load(*args, **kwargs) if hasattr(super(), "load") else None
            device_to = kwargs.get("device_to", args[0] if args else None)
            for name, module in self.model.named_modules():
                if not getattr(module, "_is_quantized", False):
                    continue
                wkey = name + ".weight"
                if wkey not in self.patches:
                    continue
                if hasattr(module, "weight_function"):
                    module.weight_function = [f for f in module.weight_function
                                              if type(f).__name__ != "LowVramPatch"]
                if Int8TensorwiseOps.dynamic_lora:
                    module.weight_lowvram_function = None
                    self.patch_weight_to_device(wkey, device_to=device_to)
                else:
                    module.weight_lowvram_function = INT8LowVramPatch(
                        wkey, self.patches, module, getattr(Int8TensorwiseOps, "lora_mode", "None"))
            return res

        def unpatch_model(self, device_to=None, unpatch_weights=True):
            if unpatch_weights:
                for module in self.model.modules():
                    if hasattr(module, "lora_patches"):
                        module.lora_patches = []
            return super().unpatch_model(device_to, unpatch_weights)

        def clone(self, *args, **kwargs):
            """Clone as an INT8-aware patcher: a patcher of another class is
            re-typed to a subclass mixing this one in for the duration of the
            base clone, so the copy keeps the INT8 LoRA routing
            (int8_quant.py:1103-1135)."""
            src_cls = self.__class__
            if src_cls is INT8ModelPatcher:
                return super().clone(*args, **kwargs)
            mixed = src_cls if issubclass(src_cls, INT8ModelPatcher) else \
                type(f"INT8_{src_cls.__name__}", (INT8ModelPatcher, src_cls), {})
            self.__class__ = mixed
            try:
                if (hasattr(self, "is_dynamic") and not self.is_dynamic()
                        and getattr(self, "cached_patcher_init", None) is None):
                    self.cached_patcher_init = (lambda *a, **kw: self, ())
                n = super().clone(*args, **kwargs)
            finally:
                self.__class__ = src_cls
            disable_dynamic = args[0] if args else kwargs.get("disable_dynamic", False)
            if disable_dynamic and not isinstance(n, INT8ModelPatcher):
                n.__class__ = type(f"INT8_{n.__class__.__name__}", (INT8ModelPatcher, n.__class__), {})
            return n
