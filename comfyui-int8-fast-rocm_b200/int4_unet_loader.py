"""``Load Diffusion Model Int4`` node (reference: int4_unet_loader.py).
Loads a diffusion model with ``Int4ConvRotOps``: ``convrot_w4a4``
checkpoints (per-layer groupsize from their ``comfy_quant`` metadata, which
is bridged from the safetensors header when stored there), or quantisation
of a high-precision model while loading; pre-loaded LoRAs are baked before
quantisation and the model is wrapped in ``Int4ModelPatcher``."""
from __future__ import annotations

import logging

import torch
import folder_paths
import comfy.sd
import comfy.utils

from .int4_quant import CONVROT_W4A4_GROUP_SIZE, MODEL_TYPE_EXCLUSIONS, Int4ConvRotOps, Int4ModelPatcher
from .loader_common import (COMPUTE_DTYPES, bridge_header_quant_metadata, group_pre_loras, normalize_lora_mode,
                            pre_lora_list, report_unmatched, stash_metadata)

INT4_MODEL_TYPES = ["flux2", "z-image", "ideogram4", "chroma", "krea2", "wan", "ltx2", "qwen", "ernie", "anima",
                    "hidream o1", "boogu"]


def bridge_convrot_w4a4_metadata(sd, metadata) -> int:
    """``<layer>.comfy_quant`` markers for the ``convrot_w4a4`` layers listed in
    the safetensors header (int4_unet_loader.py:82-130); see
    :func:`loader_common.bridge_header_quant_metadata`."""
    return bridge_header_quant_metadata(sd, metadata, ("convrot_w4a4",), "INT4 ConvRot")


class UNetLoaderINT4ConvRot:
    """Load INT4 ConvRot W4A4 diffusion models running on the B200 packed-int4
    tensor-core GEMM."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "unet_name": (folder_paths.get_filename_list("diffusion_models"),),
                "weight_dtype": (["default", "fp16", "bf16", "fp32"],
                                 {"tooltip": "Compute dtype of the activation rotation/quantisation and the "
                                             "output. Default follows the activation dtype."}),
                "model_type": (INT4_MODEL_TYPES,
                               {"tooltip": "Only used for on-the-fly quantisation, to keep sensitive layers in "
                                           "high precision."}),
                "on_the_fly_quantization": ("BOOLEAN", {"default": False,
                                                        "tooltip": "Quantise a high-precision model to INT4 "
                                                                   "ConvRot W4A4 while loading."}),
                "convrot_groupsize": ("INT", {"default": CONVROT_W4A4_GROUP_SIZE, "min": 4, "max": 4096, "step": 4,
                                              "tooltip": "On-the-fly quantisation only; checkpoints carry their "
                                                         "own per-layer groupsize."}),
                "lora_mode": (["None", "Stochastic", "Dynamic"], {"default": "None"}),
            },
            "optional": {"pre_lora": ("PRE_LORA",)},
        }

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load_unet"
    CATEGORY = "loaders"
    DESCRIPTION = "Load INT4 ConvRot W4A4 models with B200 tensor-core inference."

    def load_unet(self, unet_name, model_type, on_the_fly_quantization, weight_dtype="default",
                  convrot_groupsize=CONVROT_W4A4_GROUP_SIZE, lora_mode="None", pre_lora=None):
        unet_path = folder_paths.get_full_path("diffusion_models", unet_name)
        lora_mode = normalize_lora_mode(lora_mode)
        loras = pre_lora_list(pre_lora)

        ops_cls = Int4ConvRotOps
        ops_cls.excluded_names = list(MODEL_TYPE_EXCLUSIONS.get(model_type, []))
        ops_cls.dynamic_quantize = bool(on_the_fly_quantization)
        ops_cls.convrot_groupsize = int(convrot_groupsize)
        ops_cls.compute_dtype = COMPUTE_DTYPES.get(str(weight_dtype))
        ops_cls._is_prequantized = False
        ops_cls.lora_mode = lora_mode
        ops_cls.dynamic_lora = lora_mode == "Dynamic"
        if hasattr(ops_cls, "_logged_otf"):
            delattr(ops_cls, "_logged_otf")

        sd, metadata = comfy.utils.load_torch_file(unet_path, return_metadata=True)
        bridge_convrot_w4a4_metadata(sd, metadata)

        ops_cls.lora_patches = group_pre_loras(ops_cls, sd, metadata, loras, "INT4 ConvRot") if loras else {}
        try:
            ops_cls.applied_lora_patches = set()
            model = comfy.sd.load_diffusion_model_state_dict(sd, model_options={"custom_operations": ops_cls},
                                                             metadata=metadata)
            if model is None:
                raise RuntimeError(f"INT4 ConvRot: ComfyUI could not detect a model architecture for '{unet_name}'.")
            report_unmatched(ops_cls, "INT4 ConvRot")
        finally:
            ops_cls.lora_patches = {}
            if hasattr(ops_cls, "applied_lora_patches"):
                delattr(ops_cls, "applied_lora_patches")
        if not on_the_fly_quantization and not ops_cls._is_prequantized:
            logging.warning("INT4 ConvRot: on_the_fly_quantization is off and no convrot_w4a4 layers were found; "
                            "the model loaded at its original precision.")
        model = Int4ModelPatcher.clone(model)
        stash_metadata(model, metadata, "_int4_source_metadata")
        return (model,)
