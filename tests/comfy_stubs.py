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
    return comfy


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
