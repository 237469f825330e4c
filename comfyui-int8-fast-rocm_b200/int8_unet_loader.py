"""``Load Diffusion Model Int8`` and ``Int8 Pre-Lora Loader`` nodes
(reference: int8_unet_loader.py).  Loads a diffusion model with
``Int8TensorwiseOps`` as ComfyUI's custom operations: pre-quantised
``int8_tensorwise`` / ``asym_w4a8_int8`` checkpoints load directly,
high-precision ones are quantised per layer on the fly (optionally with
ConvRot), pre-loaded LoRAs are baked before quantisation, and the result is
wrapped in ``INT8ModelPatcher``."""
from __future__ import annotations

import logging

import torch
import folder_paths
import comfy.memory_management
import comfy.model_management
import comfy.sd
import comfy.utils

from .int8_quant import INT8ModelPatcher, Int8TensorwiseOps
from .loader_common import (COMPUTE_DTYPES, group_pre_loras, normalize_lora_mode, pre_lora_list, report_unmatched,
                            stash_metadata)

# Layers kept in high precision when quantising on the fly, per model family
# (int8_unet_loader.py:101-175; the same names as the reference so existing
# workflows keep their behaviour).
INT8_MODEL_TYPE_EXCLUSIONS = {
    "flux2": ["img_in", "time_in", "guidance_in", "txt_in", "double_stream_modulation_img",
              "double_stream_modulation_txt", "single_stream_modulation"],
    "z-image": ["cap_embedder", "t_embedder", "x_embedder", "cap_pad_token", "context_refiner", "final_layer",
                "noise_refiner", "adaLN", "x_pad_token", "layers.0."],
    "chroma": ["distilled_guidance_layer", "final_layer", "img_in", "txt_in", "nerf_image_embedder", "nerf_blocks",
               "nerf_final_layer_conv", "__x0__"],
    "qwen": ["time_text_embed", "img_in", "norm_out", "proj_out", "txt_in"],
    "ernie": ["time", "x_embedder", "text_proj", "adaLN"],
    "anima": ["embed", "llm", "adaln"],
    "krea2": ["first", "last", "tmlp", "tproj", "txtfusion", "txtmlp"],
    "hidream o1": ["embed", "language_model.layers.35.mlp"],
    "boogu": ["embed", "refine", "norm_out"],
    "ideogram4": ["embed_image_indicator", "t_embedding", "proj"],
    "wan": ["patch_embedding", "text_embedding", "time_embedding", "time_projection", "head", "img_emb",
            "face_adapter", "face_encoder", "motion_encoder", "pose_patch_embedding"],
    "ltx2": ["adaln", "embedding", "patchify", "to_gate_logits", "proj_out", "model.audio", "model.video",
             "model.av", "model.patch", "model.proj", "shift"],
    "trellis2": ["input_layer", "out_layer", "t_embedder", "rope"],
    "minimax h3": ["token_refiner", "adaln", "patch_proj", "condition_proj", "final_layer"],
    "minimax h3 skip edges": ["token_refiner", "adaln", "patch_proj", "condition_proj", "final_layer",
                              "blocks.0.", "blocks.1.", "blocks.48.", "blocks.49."],
}
INT8_MODEL_TYPES = ["flux2", "z-image", "ideogram4", "chroma", "krea2", "wan", "ltx2", "qwen", "ernie", "anima",
                    "hidream o1", "boogu", "trellis2", "minimax h3", "minimax h3 skip edges"]


def _load_int8_unet_cached_patcher(unet_name, weight_dtype, model_type, on_the_fly_quantization, enable_convrot,
                                   lora_mode, pre_lora=None, disable_dynamic=False):
    """Reload factory ComfyUI calls to rebuild the model from disk."""
    return UNetLoaderINTW8A8().load_unet(unet_name, weight_dtype, model_type, on_the_fly_quantization,
                                         enable_convrot=enable_convrot, lora_mode=lora_mode, pre_lora=pre_lora,
                                         disable_dynamic=disable_dynamic)[0]


class UNetLoaderINTW8A8:
    """Load INT8 W8A8 diffusion models (pre-quantised or quantised while
    loading) running on the B200 int8 tensor-core kernels."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "unet_name": (folder_paths.get_filename_list("diffusion_models"),),
                "weight_dtype": (["default", "fp16", "bf16", "fp32"],
                                 {"tooltip": "Activation / output dtype of the INT8 linears. Default follows the "
                                             "input activation dtype."}),
                "model_type": (INT8_MODEL_TYPES,
                               {"tooltip": "Only used for on-the-fly quantisation, to keep sensitive layers in "
                                           "high precision."}),
                "on_the_fly_quantization": ("BOOLEAN", {"default": False,
                                                        "tooltip": "Quantise a high-precision model to INT8 while "
                                                                   "loading. Keep off for INT8 checkpoints."}),
                "enable_convrot": ("BOOLEAN", {"default": True,
                                               "tooltip": "ConvRot (block Hadamard) rotation before quantisation."}),
                "lora_mode": (list(("None", "Stochastic", "Dynamic")), {"default": "None",
                              "tooltip": "None/Stochastic bake LoRAs into the INT8 weight (nearest / stochastic "
                                         "rounding); Dynamic adds the low-rank branch at inference."}),
            },
            "optional": {"pre_lora": ("PRE_LORA",)},
        }

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load_unet"
    CATEGORY = "loaders"
    DESCRIPTION = "Load and quantise INT8 models with B200 tensor-core inference."

    def load_unet(self, unet_name, weight_dtype, model_type, on_the_fly_quantization, enable_convrot=False,
                  lora_mode="None", pre_lora=None, disable_dynamic=False):
        unet_path = folder_paths.get_full_path("diffusion_models", unet_name)
        lora_mode = normalize_lora_mode(lora_mode)
        loras = pre_lora_list(pre_lora)

        ops_cls = Int8TensorwiseOps
        ops_cls.excluded_names = list(INT8_MODEL_TYPE_EXCLUSIONS.get(model_type, []))
        ops_cls.dynamic_quantize = bool(on_the_fly_quantization)
        ops_cls.enable_convrot = bool(enable_convrot)
        ops_cls.use_triton = True
        ops_cls._is_prequantized = False
        ops_cls.lora_mode = lora_mode
        ops_cls.dynamic_lora = lora_mode == "Dynamic"
        ops_cls.dynamic_load_device = None
        ops_cls.compute_dtype = COMPUTE_DTYPES.get(str(weight_dtype))
        if getattr(comfy.memory_management, "aimdo_enabled", False) and (on_the_fly_quantization or loras):
            ops_cls.dynamic_load_device = comfy.model_management.get_torch_device()
        if hasattr(ops_cls, "_logged_otf"):
            delattr(ops_cls, "_logged_otf")

        sd, metadata = comfy.utils.load_torch_file(unet_path, return_metadata=True)
        from .w4a8_int8 import bridge_w4a8_metadata_to_comfy_quant
        bridge_w4a8_metadata_to_comfy_quant(sd, metadata)

        ops_cls.lora_patches = group_pre_loras(ops_cls, sd, metadata, loras, "INT8 Fast") if loras else {}
        try:
            ops_cls.applied_lora_patches = set()
            model = comfy.sd.load_diffusion_model_state_dict(sd, model_options={"custom_operations": ops_cls},
                                                             metadata=metadata, disable_dynamic=disable_dynamic)
            if model is None:
                raise RuntimeError(f"INT8 Fast: ComfyUI could not detect a model architecture for '{unet_name}'.")
            report_unmatched(ops_cls, "INT8 Fast")
        finally:
            load_dev = ops_cls.dynamic_load_device
            ops_cls.lora_patches = {}
            ops_cls.dynamic_load_device = None
            if load_dev is not None and torch.cuda.is_available():
                torch.cuda.empty_cache()
            if hasattr(ops_cls, "applied_lora_patches"):
                delattr(ops_cls, "applied_lora_patches")

        model = INT8ModelPatcher.clone(model)
        model.cached_patcher_init = (_load_int8_unet_cached_patcher,
                                     (unet_name, weight_dtype, model_type, on_the_fly_quantization, enable_convrot,
                                      lora_mode, pre_lora))
        stash_metadata(model, metadata, "_int8_source_metadata")
        return (model,)


class PreLoraLoader:
    """Collect LoRA files to bake while the INT8 model loads.  The front end
    adds ``lora_name_<i>`` / ``lora_strength_<i>`` inputs dynamically; they are
    read back from the raw prompt (int8_unet_loader.py:312-367)."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "lora_name_1": (["None"] + folder_paths.get_filename_list("loras"),),
                "lora_strength_1": ("FLOAT", {"default": 1.0, "min": -10.0, "max": 10.0, "step": 0.01}),
            },
            "hidden": {"prompt": "PROMPT", "id": "UNIQUE_ID"},
        }

    RETURN_TYPES = ("PRE_LORA",)
    FUNCTION = "load_pre_lora"
    CATEGORY = "loaders"
    DESCRIPTION = "Pre-load a LoRA to bake it during quantisation."

    @classmethod
    def VALIDATE_INPUTS(cls, **kwargs):
        return True

    def load_pre_lora(self, **kwargs):
        prompt = kwargs.get("prompt") or {}
        node_id = kwargs.get("id")
        inputs = prompt[node_id].get("inputs", {}) if (prompt and node_id and node_id in prompt) else kwargs
        loras = []

        def add(name, strength):
            strength = round(strength, 2)
            if name != "None" and strength != 0.0:
                loras.append({"lora_name": name, "lora_strength": strength})

        if "lora_name" in inputs:
            add(inputs["lora_name"], inputs.get("lora_strength", 1.0))
        i = 1
        while f"lora_name_{i}" in inputs:
            add(inputs[f"lora_name_{i}"], inputs.get(f"lora_strength_{i}", 1.0))
            i += 1
        return (loras,)
