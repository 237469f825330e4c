"""Pieces shared by the INT8 and INT4 diffusion-model loader nodes
(int8_unet_loader.py:57-244, int4_unet_loader.py:46-223): LoRA-mode and
compute-dtype arguments, and grouping of pre-loaded LoRA patches by target
layer so the custom operations can bake them while the checkpoint loads.
ComfyUI modules are imported when a loader runs."""
from __future__ import annotations

import json
import logging

import torch

COMPUTE_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}
LORA_MODES = ("None", "Stochastic", "Dynamic")


def normalize_lora_mode(lora_mode) -> str:
    """Old workflows stored a ``dynamic_lora`` boolean; unknown values mean
    "None"."""
    if isinstance(lora_mode, bool):
        return "Dynamic" if lora_mode else "None"
    lora_mode = str(lora_mode)
    return lora_mode if lora_mode in LORA_MODES else "None"


def pre_lora_list(pre_lora):
    if pre_lora is None:
        return []
    return pre_lora if isinstance(pre_lora, list) else [pre_lora]


def normalize_key(key):
    if not isinstance(key, str):
        return key
    for p in ("diffusion_model.", "model.diffusion_model.", "model.", "transformer."):
        if key.startswith(p):
            return key[len(p):]
    return key


def group_pre_loras(ops_cls, sd, metadata, loras, tag="INT8 Fast"):
    """LoRA patches of every selected file, grouped by normalised target key:
    ``{key: [(value, offset, function, strength), ...]}``.  The key map comes
    from a meta-device skeleton of the detected architecture built with
    ``ops_cls`` (its Linear skips weight allocation while
    ``skeleton_meta_init`` is set)."""
    import folder_paths
    import comfy.lora
    import comfy.lora_convert
    import comfy.model_detection
    import comfy.utils

    grouped = {}
    for lora in loras:
        name = lora.get("lora_name", "None")
        strength = lora.get("lora_strength", 1.0)
        if name == "None" or strength == 0:
            continue
        data = comfy.utils.load_torch_file(folder_paths.get_full_path("loras", name), safe_load=True)
        data = comfy.lora_convert.convert_lora(data)
        prefix = comfy.model_detection.unet_prefix_from_state_dict(sd)
        config = comfy.model_detection.model_config_from_unet(sd, prefix, metadata=metadata)
        if config is None and prefix != "":
            config = comfy.model_detection.model_config_from_unet(sd, "", metadata=metadata)
            if config is not None:
                prefix = ""
        if config is None:
            logging.warning(f"{tag}: could not detect the model type for LoRA key mapping.")
            continue
        config.custom_operations = ops_cls
        ops_cls.skeleton_meta_init = True
        try:
            skeleton = config.get_model(sd, prefix)
        finally:
            ops_cls.skeleton_meta_init = False
        key_map = comfy.lora.model_lora_keys_unet(skeleton, {})
        for k, v in comfy.lora.load_lora(data, key_map).items():
            target, offset, function = k, None, None
            if isinstance(k, tuple):
                target = k[0]
                offset = k[1] if len(k) > 1 else None
                function = k[2] if len(k) > 2 else None
            grouped.setdefault(normalize_key(target), []).append((v, offset, function, strength))
        del data
    if grouped:
        logging.info(f"{tag}: prepared {len(grouped)} layer patches for baking.")
    return grouped


def report_unmatched(ops_cls, tag):
    if not ops_cls.lora_patches:
        return set()
    unmatched = set(ops_cls.lora_patches) - getattr(ops_cls, "applied_lora_patches", set())
    if unmatched:
        logging.warning(f"{tag}: {len(unmatched)} LoRA keys were NOT matched:")
        for k in sorted(unmatched):
            logging.warning(f"  unmatched: {k}")
    return unmatched


def stash_metadata(model, metadata, attr):
    """Keep the checkpoint header on the patcher and on the inner model
    (the inner object survives ModelPatcher.clone)."""
    model._safetensors_metadata = metadata
    try:
        if model.model is not None:
            setattr(model.model, attr, metadata)
    except Exception:
        pass


# Where a checkpoint's header names a layer "blocks.0.attn" its weight may be
# stored under one of the prefixes ComfyUI checkpoints use (the key-matching
# rule of int4_unet_loader.py:82-130 and w4a8_int8.py:78-121, which existing
# checkpoints rely on): the bare name first, then these prefixes in order,
# then any unique key that ends in the layer's name.
HEADER_KEY_PREFIXES = ("", "model.", "diffusion_model.", "model.diffusion_model.")


def _find_layer_weight(layer: str, keys) -> str | None:
    for prefix in HEADER_KEY_PREFIXES:
        if f"{prefix}{layer}.weight" in keys:
            return f"{prefix}{layer}.weight"
    tail = f".{layer}.weight"
    hits = [k for k in keys if k.endswith(tail)]
    return hits[0] if len(hits) == 1 else None


def bridge_header_quant_metadata(state_dict: dict, metadata, formats, tag: str) -> int:
    """Give every layer that the safetensors header's ``_quantization_metadata``
    lists with a format in ``formats`` a ``<layer>.comfy_quant`` tensor (the
    layer's JSON entry as uint8 bytes) when the state dict has none, so the
    custom operations see the per-layer format while loading.  Returns the
    number of layers with a marker; unparsable headers and layers whose
    weight is not found are logged and skipped."""
    raw = (metadata or {}).get("_quantization_metadata")
    if raw is None:
        return 0
    try:
        layers = json.loads(raw).get("layers", {})
    except (ValueError, AttributeError) as e:
        logging.warning(f"{tag}: ignoring an unreadable _quantization_metadata header ({e})")
        return 0
    wanted = {name: entry for name, entry in layers.items()
              if isinstance(entry, dict) and entry.get("format") in formats}
    keys = set(state_dict)
    marked = 0
    for name, entry in wanted.items():
        wkey = _find_layer_weight(name, keys)
        if wkey is None:
            logging.warning(f"{tag}: header lists layer {name!r} but the checkpoint has no weight for it")
            continue
        marker = wkey[: -len("weight")] + "comfy_quant"
        if marker not in state_dict:
            state_dict[marker] = torch.frombuffer(bytearray(json.dumps(entry, separators=(",", ":")).encode()),
                                                  dtype=torch.uint8)
        marked += 1
    if marked:
        logging.info(f"{tag}: {marked} layer formats taken from the safetensors header")
    return marked
