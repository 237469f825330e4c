"""The C-ABI library: it loads without a GPU, exports every entry point the
public header declares with the argument count the ctypes binding uses, and
rejects bad arguments with a status code and a message (validation-only
calls; no kernel is launched)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "qlinear_b200.h")


def header_decls():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    decls = {}
    for m in re.finditer(r"QLIN_API\s+[\w\s\*]+?\b(qlin_\w+)\s*\(([^)]*)\)\s*;", txt):
        args = [a for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        decls[m.group(1)] = len(args)
    return decls


def test_header_lists_entry_points():
    d = header_decls()
    for name in ["qlin_quant_act_int8", "qlin_gemm_w8a8", "qlin_int4_mm", "qlin_requant_asym_w4a8"]:
        assert name in d


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._native.load()
    decls = header_decls()
    for name, nargs in decls.items():
        assert hasattr(lib, name), name
        if name in pkg._native.SIGNATURES:
            assert len(pkg._native.SIGNATURES[name]) == nargs, name
    assert set(pkg._native.exported_symbols()) <= set(decls)


def test_version_and_empty_calls(pkg):
    lib = pkg._native.load()
    assert lib.qlin_version() >= 10000
    # M == 0: nothing to do, no device touched
    assert lib.qlin_quant_act_int8(None, 0, 0, 256, 256, 0, 0, 0.0, None, None, None) == 0


def test_validation_errors_without_gpu(pkg):
    N = pkg._native
    lib = N.load()
    # bad dtype
    assert lib.qlin_quant_act_int8(None, 9, 4, 16, 16, 0, 0, 0.0, None, None, None) == N.ERR_INVALID_ARG
    assert b"x_dtype" in lib.qlin_last_error()
    # null pointers
    assert lib.qlin_quant_act_int8(None, N.BF16, 4, 16, 16, 0, 0, 0.0, None, None, None) == N.ERR_INVALID_ARG
    assert b"null" in lib.qlin_last_error()
    # ldx < K
    assert lib.qlin_rotate(None, N.BF16, 4, 64, 32, N.ROT_REGULAR, 16, 0.25, None, None) == N.ERR_INVALID_ARG
    # K not a multiple of 16 for the int8 GEMM
    assert lib.qlin_gemm_w8a8(None, None, None, None, 1, None, None, N.BF16, 4, 4, 20, None) == N.ERR_ALIGNMENT
    # int4 group other than 0/128
    assert lib.qlin_quant_act_int4(None, N.BF16, 4, 256, 256, 0, 0, 0.0, 64, 0.0, None, None, None) == \
        N.ERR_UNSUPPORTED


def test_native_error_raises(pkg):
    with pytest.raises(pkg._native.NativeError) as ei:
        pkg._native.call("qlin_quant_act_int8", None, 9, 4, 16, 16, 0, 0, 0.0, None, None, None)
    assert ei.value.code == pkg._native.ERR_INVALID_ARG


def test_product_path_has_no_cpu_fallback(pkg):
    import torch
    with pytest.raises(RuntimeError):
        pkg.ops.quant_act_int8(torch.zeros(4, 16, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError):
        pkg.ops.int_mm(torch.zeros(4, 16, dtype=torch.int8), torch.zeros(8, 16, dtype=torch.int8))


def test_package_does_not_import_oracle(pkg):
    import sys
    src_dir = os.path.join(ROOT, "comfyui-int8-fast-rocm_b200")
    for f in os.listdir(src_dir):
        if f.endswith(".py"):
            txt = open(os.path.join(src_dir, f)).read()
            assert "oracle" not in txt.replace("oracles", ""), f
