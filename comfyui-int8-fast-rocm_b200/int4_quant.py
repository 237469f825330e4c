"""INT4 ConvRot W4A4 math and the ``Int4ConvRotOps`` ComfyUI custom
operations (reference: int4_quant.py).

The forward is two launches: the fused rotate + int4 activation quantiser
(codes in int8 storage, as the reference's ``quantize_signed_int4_rowwise``)
and the tcgen05 GEMM that unpacks the packed weight nibbles in shared memory
(``triton_int4_mm`` + the float32 epilogue of ``convrot_w4a4_forward``).
"""
from __future__ import annotations

import logging

import torch
from torch import Tensor, nn
import torch.nn.functional as F

from . import library as kops  # the kernels as registered torch.library operators
from .linear_common import QuantLowVramPatch, calc_weight_entries, float_forward, init_linear, store_param
from .int8_quant import (_normalize_lora_key, _parse_comfy_quant, _pop_metadata, int8_forward_dynamic,
                         int8_forward_dynamic_per_row, rot_for_group)

CONVROT_W4A4_GROUP_SIZE = 256
_INT4_MAX = 7


def pack_int4_row_major(values: Tensor) -> Tensor:
    """(..., K) nibbles -> (..., K//2) int8; low nibble = even column
    (int4_quant.py:36-47)."""
    if values.shape[-1] % 2 != 0:
        raise ValueError(f"last dim must be even, got {values.shape[-1]}")
    lo = values[..., 0::2].to(torch.int32) & 0x0F
    hi = values[..., 1::2].to(torch.int32) & 0x0F
    return (lo | (hi << 4)).to(torch.uint8).view(torch.int8)


def unpack_int4_row_major(packed: Tensor) -> Tensor:
    """Inverse of pack_int4_row_major, signed nibbles (int4_quant.py:50-58)."""
    x32 = packed.to(torch.int32)
    lo = x32 & 0x0F
    hi = (x32 >> 4) & 0x0F
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(*packed.shape[:-1], -1).to(torch.int8)


def quantize_signed_int4_rowwise(x: Tensor):
    """Per-row symmetric int4 in x.dtype, int8 storage (int4_quant.py:65-73):
    (q [R,K] int8 in [-7,7], scales float32 [R])."""
    return kops.quant_act_int4(x.reshape(x.shape[0], -1))


def quantize_signed_int4_rowwise_packed(x: Tensor):
    """Same, packed two per byte (int4_quant.py:76-83)."""
    if x.dtype == torch.float32:
        return kops.quant_weight_int4(x)
    q, s = kops.quant_act_int4(x)
    return pack_int4_row_major(q), s


def quantize_convrot_w4a4_weight(weight: Tensor, convrot_groupsize: int = CONVROT_W4A4_GROUP_SIZE):
    """rotate_weight + packed signed int4 per row (int4_quant.py:121-134)."""
    if weight.dim() != 2:
        raise ValueError(f"ConvRot W4A4 expects a 2D weight, got shape {tuple(weight.shape)}")
    if weight.shape[-1] % convrot_groupsize != 0:
        raise ValueError(f"in_features {weight.shape[-1]} not divisible by convrot_groupsize {convrot_groupsize}")
    return kops.quant_weight_int4(weight.float(), rot_for_group(convrot_groupsize))


def quantize_int4_g128(x: Tensor, rot=None):
    """Group-128 int4 (per row and 128-wide K group) in x.dtype:
    (q int8 [R,K], scales float32 [R, K/128])."""
    return kops.quant_act_int4(x, rot, group=128)


def dequantize_convrot_w4a4_weight_full(qweight: Tensor, wscales: Tensor, convrot_groupsize: int,
                                        dtype: torch.dtype = torch.float32) -> Tensor:
    """Unpack, rescale, un-rotate (int4_quant.py:217-231)."""
    w = unpack_int4_row_major(qweight).to(torch.float32) * wscales.reshape(-1, 1).to(torch.float32)
    return kops.rotate(w, *rot_for_group(convrot_groupsize)).to(dtype)


def prepare_rotated_activation(x: Tensor, convrot_groupsize: int, compute_dtype: torch.dtype,
                               skip_rotation: bool = False):
    """Flatten + cast + rotate (int4_quant.py:255-289)."""
    orig_shape = x.shape
    if orig_shape[-1] % convrot_groupsize != 0:
        raise ValueError(f"Input K={orig_shape[-1]} not divisible by convrot_groupsize {convrot_groupsize}")
    x2d = x.reshape(-1, orig_shape[-1]).to(compute_dtype).contiguous()
    if skip_rotation:
        return x2d, orig_shape
    return kops.rotate(x2d, *rot_for_group(convrot_groupsize)), orig_shape


def convrot_w4a4_forward(x: Tensor, qweight: Tensor, wscales: Tensor, bias, convrot_groupsize: int,
                         compute_dtype: torch.dtype, skip_rotation: bool = False, qweight_unpacked=None,
                         x_rot=None, orig_shape=None) -> Tensor:
    """W4A4 ConvRot linear (int4_quant.py:292-353): fused rotate + int4
    activation quant, then the packed-int4 tcgen05 GEMM with the float32
    epilogue ``acc * x_scale * w_scale + bias`` rounded once."""
    if x_rot is None:
        orig_shape = x.shape
        if orig_shape[-1] % convrot_groupsize != 0:
            raise ValueError(f"Input K={orig_shape[-1]} not divisible by convrot_groupsize {convrot_groupsize}")
        x2d = x.reshape(-1, orig_shape[-1]).to(compute_dtype)
        rot = None if skip_rotation else rot_for_group(convrot_groupsize)
        qact, x_scale = kops.quant_act_int4(x2d, rot)
    else:
        qact, x_scale = kops.quant_act_int4(x_rot)
    in_f = orig_shape[-1]
    if in_f != qweight.shape[-1] * 2:
        raise ValueError(f"Input K={in_f} does not match packed qweight K={qweight.shape[-1] * 2}")
    out = kops.gemm_w4a4(qact, x_scale, qweight, wscales, bias, compute_dtype)
    return out.reshape(*orig_shape[:-1], wscales.shape[0])


def quantize_signed_int4_packed_with_scale(x: Tensor, scale: Tensor) -> Tensor:
    """Packed int4 with a given per-row scale, ``round(x / s)`` clamped to
    +-7 (int4_quant.py:86-93); used when baking LoRA into an int4 layer."""
    s = scale.reshape(-1, 1).float()
    q = torch.round(x.float() / s).clamp_(-_INT4_MAX, _INT4_MAX).to(torch.int8)
    return pack_int4_row_major(q)


def stochastic_round_int4_packed_delta(x: Tensor, scale: Tensor, seed: int = 0) -> Tensor:
    """Stochastic-rounding variant (int4_quant.py:96-114): floor + Bernoulli
    of the fraction, clamped to +-7.  torch's RNG stream: matches the
    reference in distribution, not element by element."""
    s = scale.reshape(-1, 1).float()
    y = x.float() / s
    fl = torch.floor(y)
    gen = torch.Generator(device=x.device)
    gen.manual_seed(seed)
    r = torch.rand(fl.shape, generator=gen, device=x.device, dtype=fl.dtype)
    q = torch.where(r < (y - fl), fl + 1, fl).clamp_(-_INT4_MAX, _INT4_MAX).to(torch.int8)
    return pack_int4_row_major(q)


def dequantize_simple_int8_rowwise(weight: Tensor, scale: Tensor, out_features: int, convrot: bool = False,
                                   convrot_groupsize: int = CONVROT_W4A4_GROUP_SIZE) -> Tensor:
    """float32 weight of an ``int8_tensorwise`` layer inside an int4 model,
    un-rotated when the layer is ConvRot (int4_quant.py:137-160)."""
    rot = rot_for_group(convrot_groupsize) if convrot else None
    return kops.dequant_int8(weight, scale.float().reshape(-1, 1) if scale.numel() == out_features else scale.float(),
                            rot)


def quantize_int8_with_scale(x: Tensor, scale: Tensor) -> Tensor:
    """int8 with a given per-row scale, ``round(x / s)`` clamped to +-127
    (int4_quant.py:1007-1015)."""
    s = scale.reshape(-1, 1).float()
    return torch.round(x.float() / s).clamp_(-127.0, 127.0).to(torch.int8)


# Layers kept in high precision when quantising on the fly, per model family
# (int4_quant.py:371-391; same names as the reference).
MODEL_TYPE_EXCLUSIONS = {
    "flux2": ["img_in", "time_in", "guidance_in", "txt_in", "double_stream_modulation_img",
              "double_stream_modulation_txt", "single_stream_modulation"],
    "z-image": ["cap_embedder", "t_embedder", "x_embedder", "cap_pad_token", "context_refiner", "final_layer",
                "noise_refiner", "adaLN", "x_pad_token", "layers.0."],
    "chroma": ["distilled_guidance_layer", "final_layer", "img_in", "txt_in", "nerf_image_embedder", "nerf_blocks",
               "nerf_final_layer_conv", "__x0__"],
    "qwen": ["time_text_embed", "img_in", "norm_out", "proj_out", "txt_in"],
    "ernie": ["time", "x_embedder", "text_proj", "adaLN"],
    "anima": ["embed", "llm"],
    "krea2": ["first", "last", "tmlp", "tproj", "txtfusion", "txtmlp"],
    "hidream o1": ["embed", "language_model.layers.35.mlp"],
    "boogu": ["embed", "refine", "norm_out"],
    "ideogram4": ["embed_image_indicator", "t_embedding", "proj"],
    "wan": ["patch_embedding", "text_embedding", "time_embedding", "time_projection", "head", "img_emb",
            "face_adapter", "face_encoder", "motion_encoder", "pose_patch_embedding"],
    "ltx2": ["adaln", "embedding", "patchify", "to_gate_logits", "proj_out", "model.audio", "model.video",
             "model.av", "model.patch", "model.proj", "shift"],
}


try:
    from comfy.ops import manual_cast, cast_bias_weight, uncast_bias_weight
    _COMFY_OPS_AVAILABLE = True
except ImportError:
    _COMFY_OPS_AVAILABLE = False


if _COMFY_OPS_AVAILABLE:

    class Int4ConvRotOps(manual_cast):
        """ComfyUI custom operations for INT4 ConvRot W4A4 (int4_quant.py:394-976)."""

        excluded_names: list = []
        dynamic_quantize = False
        compute_dtype = None
        convrot_groupsize = CONVROT_W4A4_GROUP_SIZE
        _is_prequantized = False
        _logged_otf = False
        debug_nan_check = False
        debug_skip_rotation = False
        debug_weight_only_reference = False
        lora_mode = "None"
        dynamic_lora = False
        lora_patches: dict = {}
        lora_strength = 1.0
        skeleton_meta_init = False

        @staticmethod
        def _default_compute_dtype(x: Tensor) -> torch.dtype:
            if x.dtype in (torch.float16, torch.bfloat16):
                return x.dtype
            return torch.float16

        class Linear(manual_cast.Linear):
            def __init__(self, in_features, out_features, bias=True, device=None, dtype=None):
                init_linear(self, Int4ConvRotOps, super().__init__, in_features, out_features, bias, device, dtype)
                self.register_buffer("weight_scale", None)
                self._is_quantized = False
                self._convrot_groupsize = Int4ConvRotOps.convrot_groupsize
                self._linear_dtype = "int4"
                self._use_convrot = False
                self._is_per_row = True
                self.comfy_cast_weights = False
                self._debug_name = "<unnamed>"
                self.lora_patches = []

            def reset_parameters(self):
                return None

            _normalize_lora_key = staticmethod(_normalize_lora_key)

            @staticmethod
            def _is_bias_key(key):
                return isinstance(key, str) and key.endswith(".bias")

            def _bake_pre_lora(self, tensor, key):
                """Pre-LoRA patches grouped by the loader, baked into a float
                weight or bias before quantisation (as Int8TensorwiseOps)."""
                table = Int4ConvRotOps.lora_patches or {}
                if tensor is None or tensor.dtype == torch.int8 or not table:
                    return tensor
                nk = _normalize_lora_key(key)
                patches = table.get(nk)
                if not patches:
                    return tensor
                if not hasattr(Int4ConvRotOps, "applied_lora_patches"):
                    Int4ConvRotOps.applied_lora_patches = set()
                Int4ConvRotOps.applied_lora_patches.add(nk)
                import comfy.lora
                import comfy.model_management
                dev = torch.device("cuda") if torch.cuda.is_available() else tensor.device
                tmp = tensor.to(dev).to(comfy.model_management.lora_compute_dtype(dev))
                entries = calc_weight_entries(patches, Int4ConvRotOps.lora_strength)
                return comfy.lora.calculate_weight(entries, tmp, key).to(tensor.dtype)

            def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs):
                self._debug_name = prefix
                weight_key = prefix + "weight"
                weight_tensor = self._bake_pre_lora(state_dict.pop(weight_key, None), weight_key)
                bias_tensor = self._bake_pre_lora(state_dict.pop(prefix + "bias", None), prefix + "bias")
                weight_scale = _pop_metadata(state_dict, prefix, "weight_scale")
                conf = _parse_comfy_quant(_pop_metadata(state_dict, prefix, "comfy_quant"))
                state_dict.pop(prefix + "input_scale", None)
                is_w4a4 = isinstance(conf, dict) and conf.get("format") == "convrot_w4a4"
                is_other = isinstance(conf, dict) and conf.get("format") not in (None, "convrot_w4a4")

                if weight_tensor is not None and weight_tensor.dtype == torch.int8 and is_w4a4:
                    if weight_scale is None:
                        error_msgs.append(f"{weight_key}: convrot_w4a4 weight found but weight_scale is missing")
                    else:
                        if weight_tensor.shape[-1] * 2 != self.in_features:
                            error_msgs.append(
                                f"{weight_key}: int4 weight implies in_features={weight_tensor.shape[-1] * 2}, "
                                f"but this Linear expects {self.in_features}")
                        self._is_quantized = True
                        self._convrot_groupsize = int(conf.get("convrot_groupsize", CONVROT_W4A4_GROUP_SIZE))
                        self._linear_dtype = conf.get("linear_dtype", "int4")
                        self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                        self.register_buffer("weight_scale", weight_scale.float())
                        Int4ConvRotOps._is_prequantized = True
                elif weight_tensor is not None and weight_tensor.dtype == torch.int8 and is_other:
                    if conf.get("format") == "int8_tensorwise" and weight_scale is not None:
                        per_row = bool(conf.get("per_row", weight_scale.numel() > 1))
                        self._is_quantized = True
                        self._linear_dtype = "int8_tensorwise"
                        self._use_convrot = bool(conf.get("convrot", False))
                        self._convrot_groupsize = int(conf.get("convrot_groupsize", CONVROT_W4A4_GROUP_SIZE))
                        self._is_per_row = per_row
                        self.weight = nn.Parameter(weight_tensor.contiguous(), requires_grad=False)
                        self.register_buffer("weight_scale", weight_scale.float().reshape(-1) if per_row
                                             else weight_scale.float().reshape(()))
                    else:
                        error_msgs.append(f"{weight_key}: unsupported quantisation format {conf.get('format')!r}")
                elif weight_tensor is not None and weight_tensor.dtype in (torch.float16, torch.bfloat16, torch.float32):
                    is_excluded = any(ex in prefix for ex in Int4ConvRotOps.excluded_names)
                    is_dim1 = self.in_features == 1 or self.out_features == 1 or weight_tensor.ndim == 1
                    fits = weight_tensor.shape[-1] % Int4ConvRotOps.convrot_groupsize == 0
                    if Int4ConvRotOps.dynamic_quantize and not is_excluded and not is_dim1 and fits:
                        w = weight_tensor.to("cuda", non_blocking=True).float()
                        q, s = quantize_convrot_w4a4_weight(w, Int4ConvRotOps.convrot_groupsize)
                        self.weight = nn.Parameter(q.cpu(), requires_grad=False)
                        self.register_buffer("weight_scale", s.cpu())
                        self._is_quantized = True
                        self._convrot_groupsize = Int4ConvRotOps.convrot_groupsize
                        self._linear_dtype = "int4"
                    else:
                        self._is_quantized = False
                        self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                else:
                    self._is_quantized = False
                    if weight_tensor is not None:
                        self.weight = nn.Parameter(weight_tensor, requires_grad=False)
                    else:
                        missing_keys.append(weight_key)
                self.bias = nn.Parameter(bias_tensor, requires_grad=False) if bias_tensor is not None else None

            def convert_weight(self, _weight, inplace=False):
                return self.weight if self._is_quantized else _weight

            def set_weight(self, out_weight, inplace_update=False, seed=0, return_weight=False, **kwargs):
                if not self._is_quantized:
                    value = out_weight.to(self.weight.dtype)
                elif out_weight.dtype == torch.int8:
                    value = out_weight
                else:  # a float patch result: requantised, and the scale follows it
                    value, scale = quantize_convrot_w4a4_weight(out_weight.float(), self._convrot_groupsize)
                    self.register_buffer("weight_scale", scale.to(self.weight_scale.device))
                return store_param(self, "weight", value, inplace_update, return_weight)

            def set_bias(self, out_bias, inplace_update=False, seed=0, return_weight=False, **kwargs):
                if out_bias is None:
                    return None
                return store_param(self, "bias", out_bias, inplace_update, return_weight, inplace_creates=True)

            def forward(self, x: Tensor) -> Tensor:
                need_cast = self.comfy_cast_weights or len(self.weight_function) > 0 or len(self.bias_function) > 0
                if not self._is_quantized:
                    return float_forward(self, x, need_cast, cast_bias_weight, uncast_bias_weight)

                if need_cast:
                    weight, bias, offload_stream = cast_bias_weight(
                        self, input=None, dtype=torch.int8, device=x.device, bias_dtype=x.dtype, offloadable=True)
                else:
                    weight, bias, offload_stream = self.weight, self.bias, None
                if weight.device != x.device:
                    weight = weight.to(x.device, non_blocking=True)
                if bias is not None and bias.device != x.device:
                    bias = bias.to(x.device, non_blocking=True)
                w_scale = self.weight_scale.to(x.device, non_blocking=True)
                compute_dtype = Int4ConvRotOps.compute_dtype or Int4ConvRotOps._default_compute_dtype(x)

                if self._linear_dtype == "int8_tensorwise":
                    x2d = x.reshape(-1, x.shape[-1]).to(compute_dtype)
                    rot = rot_for_group(self._convrot_groupsize) if self._use_convrot else None
                    if self._is_per_row:
                        y = int8_forward_dynamic_per_row(x2d, weight, w_scale, bias, compute_dtype, rot)
                    else:
                        y = int8_forward_dynamic(x2d, weight, w_scale, bias, compute_dtype, rot)
                    y = y.reshape(*x.shape[:-1], weight.shape[0])
                    x_l = kops.rotate(x2d, *rot) if (self.lora_patches and rot is not None) else x2d
                else:
                    y = convrot_w4a4_forward(x, weight, w_scale, bias, self._convrot_groupsize, compute_dtype,
                                             skip_rotation=Int4ConvRotOps.debug_skip_rotation)
                    x_l = None
                    if self.lora_patches:
                        x_l, _ = prepare_rotated_activation(x, self._convrot_groupsize, compute_dtype,
                                                            Int4ConvRotOps.debug_skip_rotation)
                if self.lora_patches:
                    y2 = y.reshape(-1, y.shape[-1])
                    for lora_down, lora_up, lora_start, lora_size in self.lora_patches:
                        lD = lora_down.to(x.device, non_blocking=True)
                        lU = lora_up.to(x.device, non_blocking=True)
                        ly = F.linear(F.linear(x_l.to(lD.dtype), lD), lU)
                        if lora_start is not None:
                            y2[:, lora_start:lora_start + lora_size] = (
                                y2[:, lora_start:lora_start + lora_size] + ly.to(y2.dtype))
                        else:
                            y2 = y2 + ly.to(y2.dtype)
                    y = y2.reshape(y.shape)
                if Int4ConvRotOps.debug_nan_check and not torch.isfinite(y).all():
                    logging.error(f"INT4 ConvRot DEBUG: NaN/Inf output at layer '{self._debug_name}'")
                if need_cast:
                    uncast_bias_weight(self, weight, bias, offload_stream)
                return y

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
# LoRA on INT4 ConvRot models: low-VRAM patch callable and the model patcher
# =============================================================================

try:
    import comfy.model_patcher as _comfy_model_patcher
    import comfy.lora as _comfy_lora
    import comfy.utils as _comfy_utils
    _COMFY_PATCHER_AVAILABLE = _COMFY_OPS_AVAILABLE
except ImportError:
    _COMFY_PATCHER_AVAILABLE = False


def bake_int4_layer_weight(module, source, delta_fn, stochastic=False, seed=0):
    """Bake a float-space patch into an INT4 model's quantised layer
    (int4_quant.py:1165-1195): dequantise (+ un-rotate), apply ``delta_fn``,
    re-rotate, requantise with the layer's ORIGINAL scale (int4: packed,
    +-7; int8_tensorwise: +-127)."""
    group = getattr(module, "_convrot_groupsize", CONVROT_W4A4_GROUP_SIZE)
    wscale = module.weight_scale.to(source.device)
    if module._linear_dtype == "int8_tensorwise":
        use_rot = bool(getattr(module, "_use_convrot", False))
        w = dequantize_simple_int8_rowwise(source, wscale, source.shape[0], convrot=use_rot, convrot_groupsize=group)
        w = delta_fn(w)
        if use_rot:
            w = kops.rotate(w.float().contiguous(), *rot_for_group(group))
        return quantize_int8_with_scale(w, wscale)
    w = dequantize_convrot_w4a4_weight_full(source, wscale, group, dtype=torch.float32)
    w = kops.rotate(delta_fn(w).float().contiguous(), *rot_for_group(group))
    if stochastic:
        return stochastic_round_int4_packed_delta(w, wscale, seed)
    return quantize_signed_int4_packed_with_scale(w, wscale)


if _COMFY_PATCHER_AVAILABLE:
    from .int8_quant import _dynamic_lora_entries

    def _managed(module):
        return getattr(module, "_is_quantized", False) and \
            getattr(module, "_linear_dtype", None) in ("int4", "int8_tensorwise")

    class Int4LowVramPatch(QuantLowVramPatch):
        """Low-VRAM LoRA on an INT4 model layer as ComfyUI streams it in
        (int4_quant.py:1018-1060)."""

        def apply(self, weight, patches):
            stochastic = self.lora_mode == "Stochastic"
            return bake_int4_layer_weight(
                self.module, weight,
                lambda w: _comfy_lora.calculate_weight(patches, w, self.key, intermediate_dtype=w.dtype),
                stochastic=stochastic, seed=_comfy_utils.string_to_seed(self.key) if stochastic else 0)

    class Int4ModelPatcher(_comfy_model_patcher.ModelPatcher):
        """ModelPatcher routing LoRA on INT4 ConvRot (and stray
        int8_tensorwise) layers through bake-in or dynamic paths
        (int4_quant.py:1118-1300)."""

        def _managed_module(self, key):
            try:
                module = _comfy_utils.get_attr(self.model, key.rsplit(".", 1)[0])
            except AttributeError:
                return None
            return module if _managed(module) else None

        def patch_weight_to_device(self, key, device_to=None, inplace_update=False, return_weight=False,
                                   force_cast=False):
            if key not in self.patches and not force_cast:
                return super().patch_weight_to_device(key, device_to, inplace_update, return_weight, force_cast)
            module = self._managed_module(key)
            if module is None:
                return super().patch_weight_to_device(key, device_to, inplace_update, return_weight, force_cast)
            if Int4ConvRotOps.Linear._is_bias_key(key):
                return _comfy_utils.get_attr(self.model, key) if return_weight else None
            patches = self.patches.get(key, [])
            if not Int4ConvRotOps.dynamic_lora:
                current = _comfy_utils.get_attr(self.model, key)
                if key not in self.backup:
                    import collections
                    Backup = collections.namedtuple("Dimension", ["weight", "inplace_update"])
                    self.backup[key] = Backup(weight=current.to(device=self.offload_device, copy=inplace_update),
                                              inplace_update=inplace_update)
                    source = current
                else:
                    source = self.backup[key].weight
                stochastic = getattr(Int4ConvRotOps, "lora_mode", "None") == "Stochastic"
                patched = bake_int4_layer_weight(
                    module, source.to("cuda"), lambda w: _comfy_lora.calculate_weight(patches, w, key),
                    stochastic=stochastic, seed=_comfy_utils.string_to_seed(key) if stochastic else 0)
                patched = patched.to(current.device)
                if return_weight:
                    return patched
                if inplace_update:
                    current.data.copy_(patched)
                else:
                    _comfy_utils.set_attr(self.model, key, nn.Parameter(patched, requires_grad=False))
                return None
            weight = _comfy_utils.get_attr(self.model, key)
            cache_key = tuple(id(p[1]) for p in patches)
            if getattr(module, "_lora_cache_key", None) != cache_key:
                group = getattr(module, "_convrot_groupsize", CONVROT_W4A4_GROUP_SIZE)
                rotated = bool(getattr(module, "_use_convrot", False)) \
                    if module._linear_dtype == "int8_tensorwise" else True
                rot = rot_for_group(group) if rotated else None
                device = weight.device if weight is not None else self.offload_device
                entries = _dynamic_lora_entries(module, patches, rot, lambda k: k % group == 0)
                module.lora_patches = [(d.to(device), u.to(device), s0, sz) for d, u, s0, sz in entries]
                module._lora_cache_key = cache_key
            return weight if return_weight else None

        def load(self, *args, **kwargs):
            if not Int4ConvRotOps.dynamic_lora:
                for k in list(self.backup):
                    if k in self.patches and self._managed_module(k) is not None:
                        bk = self.backup.pop(k)
                        if bk.inplace_update:
                            _comfy_utils.get_attr(self.model, k).data.copy_(bk.weight)
                        else:
                            _comfy_utils.set_attr(self.model, k, bk.weight)
            for k in [k for k in self.backup if k not in self.patches]:
                bk = self.backup.pop(k)
                if bk.inplace_update:
                    _comfy_utils.get_attr(self.model, k).data.copy_(bk.weight)
                else:
                    _comfy_utils.set_attr(self.model, k, bk.weight)
            for name, module in self.model.named_modules():
                if getattr(module, "lora_patches", None):
                    if not Int4ConvRotOps.dynamic_lora or (name + ".weight") not in self.patches:
                        module.lora_patches = []
            res = super().load(*args, **kwargs) if hasattr(super(), "load") else None
            device_to = kwargs.get("device_to", args[0] if args else None)
            for name, module in self.model.named_modules():
                if not _managed(module) or (name + ".weight") not in self.patches:
                    continue
                wkey = name + ".weight"
                if hasattr(module, "weight_function"):
                    module.weight_function = [f for f in module.weight_function
                                              if type(f).__name__ != "LowVramPatch"]
                if Int4ConvRotOps.dynamic_lora:
                    module.weight_lowvram_function = None
                    self.patch_weight_to_device(wkey, device_to=device_to)
                else:
                    module.weight_lowvram_function = Int4LowVramPatch(
                        wkey, self.patches, module, getattr(Int4ConvRotOps, "lora_mode", "None"))
            return res

        def unpatch_model(self, device_to=None, unpatch_weights=True):
            if unpatch_weights:
                for module in self.model.modules():
                    if hasattr(module, "lora_patches"):
                        module.lora_patches = []
            return super().unpatch_model(device_to, unpatch_weights)

        def clone(self, *args, **kwargs):
            """Clone as an INT4-aware patcher (same scheme as INT8ModelPatcher.clone)."""
            src_cls = self.__class__
            if src_cls is Int4ModelPatcher:
                return super().clone(*args, **kwargs)
            mixed = src_cls if issubclass(src_cls, Int4ModelPatcher) else \
                type(f"INT4_{src_cls.__name__}", (Int4ModelPatcher, src_cls), {})
            self.__class__ = mixed
            try:
                n = super().clone(*args, **kwargs)
            finally:
                self.__class__ = src_cls
            return n
