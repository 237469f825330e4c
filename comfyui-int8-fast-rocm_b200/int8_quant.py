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

from . import ops

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
    return ops.requant_int8(_rows2d(x.float()), scale).reshape(x.shape)


def quantize_int8_tensorwise(x: Tensor):
    """(q, scale) with one absmax/127 scale for the whole tensor."""
    scale = (x.abs().max().float() / 127.0).clamp(min=1e-30)
    return quantize_int8(x, scale), scale


def quantize_int8_axiswise(x: Tensor, dim: int):
    """Per-axis absmax int8 along the last axis (dim=-1 for activations,
    dim=1 for a 2-D weight)."""
    if dim not in (-1, x.dim() - 1):
        raise ValueError("quantize_int8_axiswise supports the last axis (dim=-1, or dim=1 for 2-D weights)")
    q, s = ops.quant_act_int8(_rows2d(x))
    return q.reshape(x.shape), s.reshape(tuple(x.shape[:-1]) + (1,))


def dequantize(q: Tensor, scale) -> Tensor:
    """q.float() * scale (float32)."""
    return ops.dequant_int8(_rows2d(q), scale).reshape(q.shape)


def stochastic_round_int8_delta(x: Tensor, scale, seed: int = 0) -> Tensor:
    """Stochastic int8 rounding of x/scale (int8_quant.py:80-106): floor +1
    with probability equal to the fraction.  The kernel's counter-based RNG
    draws differ from torch.Generator's stream (same law)."""
    return ops.requant_int8(_rows2d(x.float()), scale, stochastic=True, seed=seed).reshape(x.shape)


# --- W8A8 forward (int8_quant.py:113-164) ------------------------------------


@torch.no_grad()
def int8_forward_dynamic(x: Tensor, weight: Tensor, weight_scale, bias, compute_dtype, rot=None) -> Tensor:
    """Per-token activation quant + W8A8 GEMM with a scalar weight scale."""
    xq, xs = ops.quant_act_int8(x, rot)
    if not isinstance(weight_scale, torch.Tensor):
        weight_scale = torch.tensor([float(weight_scale)], dtype=torch.float32, device=x.device)
    return ops.gemm_w8a8(xq, xs, weight, weight_scale, bias, compute_dtype, per_row=False)


@torch.no_grad()
def int8_forward_dynamic_per_row(x: Tensor, weight: Tensor, weight_scale: Tensor, bias, compute_dtype,
                                 rot=None) -> Tensor:
    """Per-token activation quant + W8A8 GEMM with per-row weight scales."""
    xq, xs = ops.quant_act_int8(x, rot)
    return ops.gemm_w8a8(xq, xs, weight, weight_scale, bias, compute_dtype, per_row=True)


def lowvram_patch_int8(weight: Tensor, scale, convrot_groupsize, delta_fn, stochastic=False, seed=0) -> Tensor:
    """INT8LowVramPatch.__call__ / bake-in path (int8_quant.py:809-843,
    881-941) on the kernels: dequant (+ un-rotate) -> ``delta_fn`` (the
    float-space patch, e.g. comfy.lora.calculate_weight) -> re-rotate ->
    requantise with the ORIGINAL scale (RNE or stochastic)."""
    rot = rot_for_group(convrot_groupsize) if convrot_groupsize else None
    w = ops.dequant_int8(weight, scale, rot)
    w = delta_fn(w)
    return ops.requant_int8(w, scale, rot, stochastic=stochastic, seed=seed)


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
                if getattr(Int8TensorwiseOps, "skeleton_meta_init", False):
                    nn.Module.__init__(self)
                    self.in_features = in_features
                    self.out_features = out_features
                    kw = {"device": "meta"}
                    if dtype is not None:
                        kw["dtype"] = dtype
                    self.weight = nn.Parameter(torch.empty((out_features, in_features), **kw), requires_grad=False)
                    self.bias = nn.Parameter(torch.empty((out_features,), **kw), requires_grad=False) if bias else None
                else:
                    super().__init__(in_features, out_features, bias, device, dtype)
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
                q, s = ops.quant_weight_int8(w, rot)
                self.weight = nn.Parameter(q.cpu(), requires_grad=False)
                self.register_buffer("weight_scale", s.cpu())
                self._weight_scale_scalar = None
                self._is_quantized = True
                self._is_per_row = True

            def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs):
                weight_key = prefix + "weight"
                bias_key = prefix + "bias"
                weight_scale = _pop_metadata(state_dict, prefix, "weight_scale")
                conf = _parse_comfy_quant(_pop_metadata(state_dict, prefix, "comfy_quant"))
                weight_tensor = state_dict.pop(weight_key, None)
                bias_tensor = state_dict.pop(bias_key, None)
                state_dict.pop(prefix + "input_scale", None)

                if isinstance(conf, dict) and conf.get("convrot", False):
                    self._use_convrot = True
                    Int8TensorwiseOps.enable_convrot = True
                    if "convrot_groupsize" in conf:
                        self._convrot_groupsize = int(conf["convrot_groupsize"])

                w4a8_handled = False
                if isinstance(conf, dict) and conf.get("format") == "asym_w4a8_int8":
                    if weight_tensor is None or weight_tensor.dtype != torch.int8:
                        logging.warning(f"W4A8: {weight_key} missing packed int8 weight, skipping")
                    else:
                        codebook = _pop_metadata(state_dict, prefix, "weight_codebook")
                        s_channel = _pop_metadata(state_dict, prefix, "weight_s_channel")
                        s_rel = _pop_metadata(state_dict, prefix, "weight_s_rel")
                        if codebook is None or s_channel is None or s_rel is None:
                            logging.warning(f"W4A8: {weight_key} missing codebook/s_channel/s_rel, skipping")
                        else:
                            self._is_w4a8 = True
                            self._w4a8_group_size = int(conf.get("group_size", 16))
                            self._w4a8_codebook = codebook
                            self._w4a8_s_channel = s_channel
                            self._w4a8_s_rel = s_rel
                            self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                            self._is_quantized = True
                            self._is_per_row = True
                            Int8TensorwiseOps._is_prequantized = True
                            w4a8_handled = True
                            weight_tensor = None

                if weight_tensor is not None:
                    if weight_tensor.dtype == torch.int8 and weight_scale is not None:
                        self._is_quantized = True
                        self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                        Int8TensorwiseOps._is_prequantized = True
                        per_row_hint = bool(conf["per_row"]) if isinstance(conf, dict) and "per_row" in conf else None
                        if isinstance(weight_scale, torch.Tensor):
                            if weight_scale.numel() == 1:
                                self.register_buffer("weight_scale", weight_scale.float().reshape(1))
                                self._is_per_row = False if per_row_hint is None else per_row_hint
                            elif weight_scale.dim() == 2 and weight_scale.shape[1] == 1:
                                self.register_buffer("weight_scale", weight_scale.float())
                                self._is_per_row = True if per_row_hint is None else per_row_hint
                            else:
                                self.register_buffer("weight_scale", weight_scale.float())
                                self._is_per_row = False if per_row_hint is None else per_row_hint
                        else:
                            self.register_buffer("weight_scale", torch.tensor([float(weight_scale)]))
                            self._is_per_row = False if per_row_hint is None else per_row_hint
                    elif weight_tensor.dtype in (torch.float16, torch.bfloat16, torch.float32):
                        is_excluded = any(ex in prefix for ex in Int8TensorwiseOps.excluded_names)
                        is_dim1 = self.in_features == 1 or self.out_features == 1 or weight_tensor.ndim == 1
                        if Int8TensorwiseOps.dynamic_quantize and not is_excluded and not is_dim1:
                            if not hasattr(Int8TensorwiseOps, "_logged_otf"):
                                logging.info(
                                    f"INT8 Fast: Quantizing on-the-fly (ConvRot: {Int8TensorwiseOps.enable_convrot})")
                                Int8TensorwiseOps._logged_otf = True
                            self._otf_quantize(weight_tensor)
                        else:
                            self._is_quantized = False
                            self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                    else:
                        self._is_quantized = False
                        self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                elif not w4a8_handled:
                    missing_keys.append(weight_key)

                self.bias = nn.Parameter(bias_tensor, requires_grad=False) if bias_tensor is not None else None
                if self.weight is not None:
                    self.weight_comfy_model_dtype = self.weight.dtype
                if self.weight_scale is not None:
                    self.weight_scale_comfy_model_dtype = self.weight_scale.dtype
                if self.bias is not None:
                    self.bias_comfy_model_dtype = self.bias.dtype

            def _get_weight_scale(self):
                return self.weight_scale

            def convert_weight(self, _weight, inplace=False):
                if not self._is_quantized:
                    return _weight
                return self.weight

            def set_weight(self, out_weight, inplace_update=False, seed=0, return_weight=False, **kwargs):
                if not self._is_quantized:
                    new_weight = out_weight.to(self.weight.dtype)
                elif out_weight.dtype == torch.int8:
                    new_weight = out_weight
                else:  # a float patch result: requantise with the layer's scale
                    new_weight = quantize_int8(out_weight, self._get_weight_scale().to(out_weight.device))
                if return_weight:
                    return new_weight
                if inplace_update:
                    self.weight.data.copy_(new_weight)
                else:
                    self.weight = nn.Parameter(new_weight, requires_grad=False)

            def set_bias(self, out_bias, inplace_update=False, seed=0, return_weight=False, **kwargs):
                if out_bias is None:
                    return None
                if return_weight:
                    return out_bias
                if inplace_update:
                    if self.bias is not None:
                        self.bias.data.copy_(out_bias)
                else:
                    self.bias = nn.Parameter(out_bias, requires_grad=False)

            # -- forward ----------------------------------------------------
            def _w4a8_int8_weight(self, weight):
                """asym_w4a8_int8 -> per-channel int8, computed once per device
                by the fused dequant+requant kernel and cached (the reference
                recomputes it every call, int8_quant.py:679-687)."""
                key = (weight.device, weight.data_ptr())
                hit = self._w4a8_cache.get(key)
                if hit is None:
                    hit = ops.requant_asym_w4a8(weight, self._w4a8_codebook, self._w4a8_s_channel,
                                                self._w4a8_s_rel, self._w4a8_group_size)
                    self._w4a8_cache = {key: hit}
                return hit

            def forward(self, x: Tensor) -> Tensor:
                need_cast = self.comfy_cast_weights or len(self.weight_function) > 0 or len(self.bias_function) > 0
                if not self._is_quantized:
                    if need_cast:
                        weight, bias, offload_stream = cast_bias_weight(self, x, offloadable=True)
                        out = F.linear(x, weight, bias)
                        uncast_bias_weight(self, weight, bias, offload_stream)
                        return out
                    if x.device != self.weight.device or x.dtype != self.weight.dtype:
                        weight = self.weight.to(device=x.device, dtype=x.dtype)
                        bias = self.bias.to(device=x.device, dtype=x.dtype) if self.bias is not None else None
                        return F.linear(x, weight, bias)
                    return F.linear(x, self.weight, self.bias)

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

                if self._is_per_row:
                    y = int8_forward_dynamic_per_row(x_2d, weight, w_scale, bias, compute_dtype, rot)
                else:
                    y = int8_forward_dynamic(x_2d, weight, w_scale, bias, compute_dtype, rot)

                if self.lora_patches:
                    # dynamic LoRA (int8_quant.py:718-729): down-projection of
                    # the (rotated) activation, up-projection, added to y
                    x_l = ops.rotate(x_2d, *rot) if rot is not None else x_2d
                    for lora_down, lora_up, lora_start, lora_size in self.lora_patches:
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
