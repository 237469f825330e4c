"""ctypes binding of libqlinear_b200.so (the C ABI declared in
include/qlinear_b200.h).

The shared library sits next to this file (built by build_native.py).  There
is no fallback: if it is missing, or the device is not an sm_100 GPU, every
kernel call raises.  Loading the library needs no GPU, so the symbol table
can be inspected on a CPU-only host.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libqlinear_b200.so")

# status codes / enums (mirror include/qlinear_b200.h)
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_ALIGNMENT, ERR_CUDA, ERR_NO_DEVICE = range(6)
BF16, F16, F32, I8, I32 = range(5)
ROT_NONE, ROT_REGULAR, ROT_SYLVESTER = range(3)
WSCALE_TENSOR, WSCALE_ROW = 0, 1
ROUND_NEAREST, ROUND_STOCHASTIC = 0, 1
NORM_NONE, NORM_LAYER, NORM_RMS = range(3)

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_U64 = ctypes.c_uint64

# name -> argtypes (restype int for all but qlin_last_error)
SIGNATURES = {
    "qlin_version": [],
    "qlin_set_device": [_I],
    "qlin_device_error": [_P, _P],
    "qlin_set_wait_limit": [_U64],
    "qlin_selftest_wait_timeout": [_I, _P],
    "qlin_selftest_gemm_stall": [_P, _P, _P, _P, _P, _L, _L, _L, _L, _P],
    "qlin_quant_act_int8": [_P, _I, _L, _L, _L, _I, _I, _F, _P, _P, _P],
    "qlin_quant_act_int8_norm": [_P, _I, _L, _L, _L, _I, _F, _P, _P, _L, _P, _L, _L, _I, _I, _F, _P, _P, _P],
    "qlin_quant_act_int8_cat": [_P, _L, _L, _P, _L, _L, _I, _L, _I, _I, _F, _P, _P, _P],
    "qlin_qk_norm_rope": [_P, _I, _L, _L, _I, _I, _P, _P, _F, _P, _P, _L, _P],
    "qlin_quant_act_int4": [_P, _I, _L, _L, _L, _I, _I, _F, _I, _F, _P, _P, _P],
    "qlin_rotate": [_P, _I, _L, _L, _L, _I, _I, _F, _P, _P],
    "qlin_situ": [_P, _I, _L, _L, _L, _P, _P],
    "qlin_quant_act_int8_situ": [_P, _I, _L, _L, _L, _I, _I, _F, _P, _P, _P],
    "qlin_gemm_w8a8": [_P, _P, _P, _P, _I, _P, _P, _I, _L, _L, _L, _P],
    "qlin_gemm_w8a8_splitk_scratch": [_L, _L, _L, _P],
    "qlin_gemm_w8a8_splitk": [_P, _P, _P, _P, _I, _P, _P, _I, _L, _L, _L, _P, _U64, _P],
    "qlin_gemm_w8a8_splitk_noalloc": [_P, _P, _P, _P, _I, _P, _P, _I, _L, _L, _L, _P],
    "qlin_gemm_w8a8_fused": [_P, _P, _P, _P, _I, _P, _P, _I, _L, _L, _L, _L, _P, _L, _P, _L, _L, _P],
    "qlin_gemm_w8a8_fused_segments": [_P, _P, _P, _P, _I, _P, _P, _I, _L, _L, _L, _L, _P, _L, _P, _L, _L,
                                      _L, _L, _L, _L, _L, _L, _P],
    "qlin_gemm_w8a8_allgather": [_P, _P, _P, _P, _I, _P, _P, _I, _L, _L, _I, _L, _L, _L, _P],
    "qlin_int_mm": [_P, _P, _P, _L, _L, _L, _P],
    "qlin_int4_mm": [_P, _P, _P, _L, _L, _L, _P],
    "qlin_gemm_w4a4": [_P, _P, _P, _P, _P, _P, _I, _L, _L, _L, _P],
    "qlin_gemm_w4a8_g128": [_P, _P, _P, _P, _P, _P, _I, _L, _L, _L, _P],
    "qlin_gemm_w4a4_g128": [_P, _P, _P, _P, _P, _P, _I, _L, _L, _L, _P],
    "qlin_quant_weight_int8": [_P, _I, _L, _L, _I, _I, _F, _P, _P, _P],
    "qlin_quant_weight_int4": [_P, _I, _L, _L, _I, _I, _F, _I, _P, _P, _P],
    "qlin_requant_asym_w4a8": [_P, _P, _P, _P, _I, _L, _L, _P, _P, _P],
    "qlin_dequant_asym_w4a8": [_P, _P, _P, _P, _I, _L, _L, _P, _P],
    "qlin_dequant_int8": [_P, _P, _I, _L, _L, _I, _I, _F, _P, _P],
    "qlin_requant_int8": [_P, _P, _I, _L, _L, _I, _I, _F, _I, _U64, _P, _P],
}


class NativeError(RuntimeError):
    """A libqlinear_b200 entry point returned an error status."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def load():
    """Load the shared library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python comfyui-int8-fast-rocm_b200/build_native.py` (nvcc, sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
            lib.qlin_last_error.argtypes = []
            lib.qlin_last_error.restype = ctypes.c_char_p
            _lib = lib
    return _lib


def call(name, *args):
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.qlin_last_error()
        raise NativeError(name, rc, msg.decode("utf-8", "replace") if msg else "")
    return rc


def exported_symbols():
    return ["qlin_last_error"] + list(SIGNATURES)
