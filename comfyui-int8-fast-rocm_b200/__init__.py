"""INT8/INT4 quantized-linear node pack for ComfyUI, B200 (sm_100a) native.

Drop-in for the quantized-linear hot path of ComfyUI-INT8-Fast: the same
operator surface (``Int8TensorwiseOps`` / ``Int4ConvRotOps`` custom
operations, the ``int8_tensorwise`` / ``convrot_w4a4`` / ``asym_w4a8_int8``
weight formats, the INT8/INT4 UNet loader nodes and the module-level kernel
functions ``triton_int8_linear`` & co.), backed by hand-written CUDA kernels
in ``libqlinear_b200.so`` (tcgen05 int8 tensor-core GEMMs, fused
rotate+quantise).  ComfyUI-specific parts register only when ComfyUI is
importable; the kernels and math functions work standalone.
"""
import logging

from . import _native  # noqa: F401
from . import ops  # noqa: F401
from . import library  # noqa: F401  (the kernels as torch.library operators, namespace qlin_b200)
from . import convrot  # noqa: F401
from . import int8_fused_kernel  # noqa: F401
from . import triton_int4_mm  # noqa: F401
from . import w4a8_int8  # noqa: F401
from . import int8_quant  # noqa: F401
from . import int4_quant  # noqa: F401
from . import tensor_parallel  # noqa: F401
from . import int8_save  # noqa: F401
from . import data_parallel  # noqa: F401

log = logging.getLogger("comfyui-int8-fast-b200")


def _register_layouts():
    """Register the ``int8_tensorwise`` layout/algorithm with ComfyUI's
    quantisation registry (same entries as the reference, __init__.py:21-69)."""
    try:
        import torch
        from comfy.quant_ops import QUANT_ALGOS, register_layout_class, QuantizedLayout
    except ImportError:
        return False

    class Int8TensorwiseLayout(QuantizedLayout):
        class Params:
            def __init__(self, scale=None, orig_dtype=None, orig_shape=None, **kwargs):
                self.scale = scale
                self.orig_dtype = orig_dtype
                self.orig_shape = orig_shape

            def clone(self):
                s = self.scale.clone() if isinstance(self.scale, torch.Tensor) else self.scale
                return Int8TensorwiseLayout.Params(scale=s, orig_dtype=self.orig_dtype, orig_shape=self.orig_shape)

        @classmethod
        def state_dict_tensors(cls, qdata, params):
            return {"": qdata, "weight_scale": params.scale}

        @classmethod
        def dequantize(cls, qdata, params):
            return qdata.float() * params.scale

    try:
        register_layout_class("Int8TensorwiseLayout", Int8TensorwiseLayout)
        QUANT_ALGOS.setdefault("int8_tensorwise", {
            "storage_t": torch.int8,
            "parameters": {"weight_scale", "input_scale"},
            "comfy_tensor_layout": "Int8TensorwiseLayout",
        })
    except Exception as e:  # registry API drift
        log.error(f"INT8 Fast B200: failed to register layouts: {e}")
        return False
    return True


_register_layouts()

Int8TensorwiseOps = getattr(int8_quant, "Int8TensorwiseOps", None)
Int4ConvRotOps = getattr(int4_quant, "Int4ConvRotOps", None)

NODE_CLASS_MAPPINGS = {}
NODE_DISPLAY_NAME_MAPPINGS = {}
try:
    from .int8_unet_loader import PreLoraLoader, UNetLoaderINTW8A8
    from .int4_unet_loader import UNetLoaderINT4ConvRot

    NODE_CLASS_MAPPINGS = {
        "OTUNetLoaderW8A8": UNetLoaderINTW8A8,
        "INT8PreLoraLoader": PreLoraLoader,
        "UNetLoaderINT4ConvRot": UNetLoaderINT4ConvRot,
    }
    NODE_DISPLAY_NAME_MAPPINGS = {
        "OTUNetLoaderW8A8": "Load Diffusion Model Int8",
        "INT8PreLoraLoader": "Int8 Pre-Lora Loader",
        "UNetLoaderINT4ConvRot": "Load Diffusion Model Int4",
    }
except ImportError:
    pass

try:
    from . import kitchen_patch  # noqa: F401  (registers int8_linear when comfy_kitchen exists)
except ImportError:
    pass

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS", "Int8TensorwiseOps", "Int4ConvRotOps", "ops", "library"]
