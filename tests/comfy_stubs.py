"""Minimal stand-ins for the ComfyUI modules the operator surface imports
(``comfy.ops.manual_cast`` & co., ``comfy.quant_ops``), so the custom
operations can be exercised without ComfyUI."""
import importlib.util
import os
import sys
import types

import torch
from torch import nn

from conftest import PKG_DIR


class _CastMixin:
    comfy_cast_weights = False

    def _init_cast(self):
        self.weight_function = []
        self.bias_function = []


class manual_cast:
    class Linear(nn.Linear, _CastMixin):
        def __init__(self, in_features, out_features, bias=True, device=None, dtype=None):
            nn.Module.__init__(self)
            self.in_features = in_features
            self.out_features = out_features
            self.weight = None
            self.bias = None
            self._init_cast()

        def reset_parameters(self):
            return None

    class GroupNorm(nn.GroupNorm):
        pass

    class LayerNorm(nn.LayerNorm):
        pass

    class Conv2d(nn.Conv2d):
        pass

    class Conv3d(nn.Conv3d):
        pass

    class ConvTranspose2d(nn.ConvTranspose2d):
        pass

    class Embedding(nn.Embedding):
        pass


def cast_bias_weight(module, input=None, dtype=None, device=None, bias_dtype=None, offloadable=False):
    dev = device if device is not None else input.device
    w = module.weight.to(device=dev, dtype=dtype if dtype is not None else input.dtype)
    b = None if module.bias is None else module.bias.to(device=dev, dtype=bias_dtype or (input.dtype if input is not None else None))
    return w, b, None


def uncast_bias_weight(module, weight, bias, offload_stream):
    return None


class QuantizedLayout:
    pass


def install():
    """Register stub comfy modules in sys.modules (idempotent)."""
    if "comfy.ops" in sys.modules and getattr(sys.modules["comfy.ops"], "_qlin_stub", False):
        return sys.modules["comfy"]
    comfy = types.ModuleType("comfy")
    comfy.__path__ = []
    ops = types.ModuleType("comfy.ops")
    ops._qlin_stub = True
    ops.manual_cast = manual_cast
    ops.cast_bias_weight = cast_bias_weight
    ops.uncast_bias_weight = uncast_bias_weight
    qo = types.ModuleType("comfy.quant_ops")
    qo.QUANT_ALGOS = {}
    qo.LAYOUTS = {}
    qo.QuantizedLayout = QuantizedLayout
    qo.register_layout_class = lambda name, cls: qo.LAYOUTS.__setitem__(name, cls)
    comfy.ops = ops
    comfy.quant_ops = qo
    sys.modules.update({"comfy": comfy, "comfy.ops": ops, "comfy.quant_ops": qo})
    _install_loader_stubs(comfy)
    return comfy


# ---------------------------------------------------------------------------
# Loader-side stand-ins: file registry, model detection, LoRA math, patcher
# ---------------------------------------------------------------------------

FILES = {}  # "<kind>/<name>" -> (state_dict, metadata)


def register_file(kind, name, sd, metadata=None):
    FILES[f"{kind}/{name}"] = (sd, metadata or {})


class ModelPatcher:
    """The parts of comfy.model_patcher.ModelPatcher the INT8/INT4 patchers use."""

    def __init__(self, model, load_device=None, offload_device=None):
        self.model = model
        self.load_device = load_device
        self.offload_device = offload_device or torch.device("cpu")
        self.patches = {}
        self.backup = {}
        self.size = 0

    def is_dynamic(self):
        return False

    def clone(self, *args, **kwargs):
        n = self.__class__(self.model, self.load_device, self.offload_device)
        n.patches = {k: list(v) for k, v in self.patches.items()}
        n.backup = self.backup
        return n

    def add_patches(self, patches, strength_patch=1.0, strength_model=1.0):
        for k, v in patches.items():
            self.patches.setdefault(k, []).append((strength_patch, v, strength_model, None, None))

    def patch_weight_to_device(self, key, device_to=None, inplace_update=False, return_weight=False,
                               force_cast=False):
        w = get_attr(self.model, key)
        out = calculate_weight(self.patches.get(key, []), w.float(), key).to(w.dtype)
        if return_weight:
            return out
        set_attr(self.model, key, nn.Parameter(out, requires_grad=False))

    def load(self, device_to=None, **kwargs):
        return None

    def unpatch_model(self, device_to=None, unpatch_weights=True):
        return None


class LoraAdapter:
    """Standard LoRA adapter: weights = (up, down, alpha, mid, dora, reshape)."""

    def __init__(self, up, down, alpha=None):
        self.weights = (up, down, alpha, None, None, None)


def calculate_weight(patches, weight, key, intermediate_dtype=None):
    """Float-space patch: tensor values are weight deltas; adapters add
    strength * alpha/rank * up @ down."""
    for p in patches:
        strength, v = p[0], p[1]
        strength_model = p[2] if len(p) > 2 else 1.0
        if isinstance(v, torch.Tensor):
            weight = weight * strength_model + strength * v.to(weight.device, weight.dtype)
        else:
            up, down, alpha = v.weights[0], v.weights[1], v.weights[2]
            rank = down.shape[0]
            sc = (alpha / rank) if alpha is not None else 1.0
            delta = (up.float() @ down.float()).to(weight.device, weight.dtype)
            weight = weight * strength_model + strength * sc * delta
    return weight


def get_attr(obj, attr):
    for name in attr.split("."):
        obj = getattr(obj, name)
    return obj


def set_attr(obj, attr, value):
    names = attr.split(".")
    for name in names[:-1]:
        obj = getattr(obj, name)
    setattr(obj, names[-1], value)


class TinyDiT(nn.Module):
    """Three linears named like a Flux block: blocks.0.qkv (256->384),
    blocks.0.proj (256->256) and img_in (256->128)."""

    def __init__(self, operations):
        super().__init__()
        self.blocks = nn.ModuleList([nn.Module()])
        self.blocks[0].qkv = operations.Linear(256, 384)
        self.blocks[0].proj = operations.Linear(256, 256)
        self.img_in = operations.Linear(256, 128)


class _Config:
    def __init__(self):
        self.custom_operations = None

    def get_model(self, sd, prefix):
        return TinyDiT(self.custom_operations)


def _install_loader_stubs(comfy):
    fp = types.ModuleType("folder_paths")
    fp.get_filename_list = lambda kind: sorted(k.split("/", 1)[1] for k in FILES if k.startswith(kind + "/"))
    fp.get_full_path = lambda kind, name: f"{kind}/{name}"
    utils = types.ModuleType("comfy.utils")

    def load_torch_file(path, return_metadata=False, safe_load=False):
        sd, md = FILES[path]
        sd = dict(sd)
        return (sd, dict(md)) if return_metadata else sd

    utils.load_torch_file = load_torch_file
    utils.get_attr = get_attr
    utils.set_attr = set_attr
    utils.string_to_seed = lambda s: sum(ord(c) for c in s) & 0xFFFFFFFF
    sd_mod = types.ModuleType("comfy.sd")

    def load_diffusion_model_state_dict(sd, model_options=None, metadata=None, disable_dynamic=False):
        model = TinyDiT(model_options["custom_operations"])
        model.load_state_dict(sd, strict=False)
        return ModelPatcher(model)

    sd_mod.load_diffusion_model_state_dict = load_diffusion_model_state_dict
    mp = types.ModuleType("comfy.model_patcher")
    mp.ModelPatcher = ModelPatcher
    lora = types.ModuleType("comfy.lora")
    lora.calculate_weight = calculate_weight
    lora.model_lora_keys_unet = lambda model, key_map: key_map
    lora.load_lora = lambda data, key_map: dict(data)
    lora_convert = types.ModuleType("comfy.lora_convert")
    lora_convert.convert_lora = lambda d: d
    md = types.ModuleType("comfy.model_detection")
    md.unet_prefix_from_state_dict = lambda sd: ""
    md.model_config_from_unet = lambda sd, prefix, metadata=None: _Config()
    mm = types.ModuleType("comfy.model_management")
    mm.lora_compute_dtype = lambda device: torch.float32
    mm.get_torch_device = lambda: torch.device("cuda")
    mem = types.ModuleType("comfy.memory_management")
    mem.aimdo_enabled = False
    for name, mod in (("utils", utils), ("sd", sd_mod), ("model_patcher", mp), ("lora", lora),
                      ("lora_convert", lora_convert), ("model_detection", md), ("model_management", mm),
                      ("memory_management", mem)):
        setattr(comfy, name, mod)
        sys.modules["comfy." + name] = mod
    sys.modules["folder_paths"] = fp


def load_package_with_comfy(name="qlin_with_comfy"):
    """A second instance of the node pack imported after the stubs exist."""
    install()
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod
