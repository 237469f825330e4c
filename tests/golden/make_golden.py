"""Generate golden vectors by running the reference node pack's own PyTorch
CPU code on seeded inputs.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/ComfyUI-INT8-Fast-ROCM

The reference's modules ``convrot``, ``int8_quant``, ``int4_quant`` and
``w4a8_int8`` are imported as a synthetic package (its ``__init__`` is NOT
executed: it registers ComfyUI nodes and runs a network self-updater) with
stub ``comfy.*`` modules.  ``comfy.ops`` is left out on purpose, so the
ComfyUI operator classes are not defined and only the module-level math
functions are used.  Inputs are generated with numpy (see ``golden_inputs``)
so that the tests can regenerate them without torch's RNG; the fixtures keep
the reference's outputs (full arrays for small cases, sha256 digests plus a
few rows for the large ones).
"""
from __future__ import annotations

import hashlib
import importlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import golden_inputs as gi  # noqa: E402


def _install_comfy_stubs():
    import torch

    comfy = types.ModuleType("comfy")
    comfy.__path__ = []
    mods = {}
    for name in ["model_patcher", "memory_management", "model_management", "lora", "utils"]:
        m = types.ModuleType("comfy." + name)
        mods[name] = m
        setattr(comfy, name, m)
        sys.modules["comfy." + name] = m

    class ModelPatcher:  # placeholder base class
        pass

    mods["model_patcher"].ModelPatcher = ModelPatcher
    mods["memory_management"].aimdo_enabled = False
    mods["memory_management"].read_tensor_file_slice_into = lambda *a, **k: False
    mods["model_management"].WINDOWS = False
    mods["model_management"].get_torch_device = lambda: torch.device("cpu")
    mods["model_management"].lora_compute_dtype = lambda d: torch.float32

    def prefetch_prepared_value(a, b, c, d, e):
        return a

    mods["lora"].prefetch_prepared_value = prefetch_prepared_value
    mods["lora"].calculate_weight = lambda patches, w, key, **kw: w
    mods["utils"].string_to_seed = lambda s: 0
    sys.modules["comfy"] = comfy


def load_reference(ref_dir):
    _install_comfy_stubs()
    pkg = types.ModuleType("refpack")
    pkg.__path__ = [ref_dir]
    sys.modules["refpack"] = pkg
    mods = {}
    for name in ["convrot", "w4a8_int8", "int8_quant", "int4_quant"]:
        mods[name] = importlib.import_module("refpack." + name)
    return mods


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref_dir):
    import torch
    from scipy.linalg import hadamard as scipy_hadamard

    torch.set_num_threads(8)
    R = load_reference(ref_dir)
    cr, i8, i4, w4 = R["convrot"], R["int8_quant"], R["int4_quant"], R["w4a8_int8"]
    out = {}

    def T(a, dt):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dt)

    def bits16(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}

    # 1. per-token int8 activation quant (int8_quant.py:49-52), small odd shapes
    for dt in ["bf16", "f16", "f32"]:
        x = gi.activation(0, 37, 256, dt, zero_row=5)
        q, s = i8.quantize_int8_axiswise(T(x, tdt[dt]), dim=-1)
        out[f"q8_{dt}_q"] = q.numpy()
        out[f"q8_{dt}_s"] = s.numpy()

    # 1b. activation quant at 4096 x 3072 (digests)
    x = gi.activation(0, 4096, 3072, "bf16")
    q, s = i8.quantize_int8_axiswise(T(x, torch.bfloat16), dim=-1)
    out["q8_c0_q_sha"] = np.array(sha(q.numpy()))
    out["q8_c0_q_rows"] = q.numpy()[:4]
    out["q8_c0_s"] = s.numpy()

    # 2. W8A8 per-row forward, CPU branch (int8_quant.py:137-164)
    for dt in ["bf16", "f16"]:
        x = gi.activation(1, 37, 256, dt)
        w = gi.weight(1, 512, 256)
        wq, ws = i8.quantize_int8_axiswise(torch.from_numpy(w), dim=1)
        out[f"w8_{dt}_wq"] = wq.numpy()
        out[f"w8_{dt}_ws"] = ws.numpy()
        b = gi.bias(1, 512, dt)
        y = i8.int8_forward_dynamic_per_row(T(x, tdt[dt]), wq, ws, T(b, tdt[dt]), tdt[dt])
        out[f"w8_{dt}_y"] = bits16(y)
        y0 = i8.int8_forward_dynamic_per_row(T(x, tdt[dt]), wq, ws, None, tdt[dt])
        out[f"w8_{dt}_y_nobias"] = bits16(y0)

    # 2b. medium W8A8 per-row with outliers, M=256 K=3072 N=384
    x = gi.activation(2, 256, 3072, "bf16")
    w = gi.weight(2, 384, 3072)
    wq, ws = i8.quantize_int8_axiswise(torch.from_numpy(w), dim=1)
    b = gi.bias(2, 384, "bf16")
    y = i8.int8_forward_dynamic_per_row(T(x, torch.bfloat16), wq, ws, T(b, torch.bfloat16), torch.bfloat16)
    out["w8m_wq_sha"] = np.array(sha(wq.numpy()))
    out["w8m_ws"] = ws.numpy()
    out["w8m_y"] = bits16(y)

    # 3. W8A8 tensorwise forward (int8_quant.py:113-133), smoke-test-like inputs
    x = gi.activation(3, 37, 256, "f16")
    wq = gi.int8_weight(3, 512, 256)
    ws = torch.tensor([0.01], dtype=torch.float32)
    b = gi.bias(3, 512, "f16")
    y = i8.int8_forward_dynamic(T(x, torch.float16), torch.from_numpy(wq), ws, T(b, torch.float16), torch.float16)
    out["w8t_y"] = bits16(y)

    # 4. rotate_activation (convrot.py:89-118)
    for g in [16, 64, 256]:
        x = gi.activation(4, 32, 1024, "bf16")
        H = cr.build_hadamard(g, device="cpu", dtype=torch.float32)
        out[f"rot_reg{g}_H"] = H.numpy()
        out[f"rot_reg{g}_y"] = bits16(cr.rotate_activation(T(x, torch.bfloat16), H, group_size=g))
    # Sylvester 128: scipy.linalg.hadamard (imported by convrot.py:12) normalised
    # the way build_hadamard normalises (float32 matrix / size**0.5).
    Hs = torch.tensor(scipy_hadamard(128), dtype=torch.float32) / (128 ** 0.5)
    out["rot_syl128_H"] = Hs.numpy()
    x = gi.activation(4, 32, 1024, "bf16")
    out["rot_syl128_y"] = bits16(cr.rotate_activation(T(x, torch.bfloat16), Hs, group_size=128))
    try:
        cr.build_hadamard(128)
        out["regular128_raises"] = np.array(0)
    except ValueError:
        out["regular128_raises"] = np.array(1)

    # 4b. rotate_weight fp32 (convrot.py:58-86)
    w = gi.weight(5, 32, 512)
    H = cr.build_hadamard(256, device="cpu", dtype=torch.float32)
    out["rotw_y"] = cr.rotate_weight(torch.from_numpy(w), H, group_size=256).numpy()

    # 5. INT4 (int4_quant.py)
    x = gi.activation(6, 37, 512, "bf16", zero_row=3)
    xr = cr.rotate_activation(T(x, torch.bfloat16), cr.build_hadamard(256, dtype=torch.float32), 256)
    q, s = i4.quantize_signed_int4_rowwise(xr)
    out["i4_xrot"] = bits16(xr)
    out["i4_q"] = q.numpy()
    out["i4_s"] = s.numpy()
    q16, s16 = i4.quantize_signed_int4_rowwise(T(gi.activation(6, 37, 512, "f16"), torch.float16))
    out["i4_f16_q"] = q16.numpy()
    out["i4_f16_s"] = s16.numpy()
    nib = gi.nibbles(7, 64, 128)
    out["i4_pack"] = i4.pack_int4_row_major(torch.from_numpy(nib)).numpy()
    out["i4_unpack"] = i4.unpack_int4_row_major(torch.from_numpy(out["i4_pack"])).numpy()
    w = gi.weight(8, 128, 512)
    pw, ps = i4.quantize_convrot_w4a4_weight(torch.from_numpy(w), convrot_groupsize=256)
    out["i4w_packed"] = pw.numpy()
    out["i4w_scale"] = ps.numpy()
    # convrot_w4a4_forward (int4_quant.py:292-353) with triton_int4_mm replaced
    # by its defined semantics (triton_int4_mm.py:4-9): a @ unpack(W).T, int32.
    x = gi.activation(9, 37, 512, "bf16")
    b = gi.bias(9, 128, "bf16")
    x_rot, shp = i4.prepare_rotated_activation(T(x, torch.bfloat16), 256, torch.bfloat16)
    qa, sa = i4.quantize_signed_int4_rowwise(x_rot)
    acc = torch._int_mm(qa, i4.unpack_int4_row_major(pw).T.contiguous())
    o = acc.to(torch.float32)
    o.mul_(sa.reshape(-1, 1))
    o.mul_(ps.reshape(1, -1))
    o.add_(T(b, torch.bfloat16).to(torch.float32).reshape(1, -1))
    out["i4fwd_acc"] = acc.numpy()
    out["i4fwd_y"] = bits16(o.to(torch.bfloat16))

    # 6. asym W4A8 (w4a8_int8.py:29-75) + requant (int8_quant.py:679-687)
    packed, codebook, s_ch, s_rel_bytes = gi.asym_w4a8(10, 96, 256, 16)
    s_rel = torch.from_numpy(s_rel_bytes).view(torch.float8_e4m3fn)
    deq = w4.dequant_asym_w4a8_to_float(torch.from_numpy(packed), torch.from_numpy(codebook),
                                        torch.from_numpy(s_ch), s_rel, 16)
    out["w4a8_deq"] = deq.numpy()
    rq, rs = i8.quantize_int8_axiswise(deq, dim=1)
    out["w4a8_q"] = rq.numpy()
    out["w4a8_s"] = rs.numpy()

    # 7. OTF weight quant with ConvRot (int8_quant.py:527-554, on CPU)
    w = gi.weight(11, 48, 512)
    wr = cr.rotate_weight(torch.from_numpy(w), cr.build_hadamard(256, dtype=torch.float32), 256)
    oq, os_ = i8.quantize_int8_axiswise(wr, dim=1)
    out["otf_q"] = oq.numpy()
    out["otf_s"] = os_.numpy()

    # 8. LoRA bake round trip (int8_quant.py:815-843): dequant -> unrotate ->
    # (+delta) -> rotate -> quantize_int8 with the original scale
    H = cr.build_hadamard(256, dtype=torch.float32)
    wf = i8.dequantize(oq, os_)
    wf = cr.rotate_weight(wf, H, 256)
    delta = torch.from_numpy(gi.weight(12, 48, 512) * np.float32(0.05))
    out["lora_unrot"] = wf.numpy()
    patched = cr.rotate_weight(wf + delta, H, 256)
    out["lora_rerot"] = patched.numpy()
    out["lora_q"] = i8.quantize_int8(patched, os_).numpy()

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes,", len(out), "arrays")

    config_scale_codes(cr, i8, scipy_hadamard)


def config_scale_codes(cr, i8, scipy_hadamard):
    """ConvRot activation codes at the W8A8 linear's full size.

    The reference rotates with a bf16 library matmul (convrot.py:114-117)
    whose float32 accumulation order is its own; the kernels (and the
    oracle) use a fixed-order butterfly.  For each case this stores the
    reference's int8 codes as a digest plus the sparse list of positions where
    they differ from the oracle's codes, and the reference's per-token scales
    in full.  The GPU test patches the kernel's codes at those positions and
    checks the digest: that proves the kernel differs from the reference at
    exactly the listed positions, which gives the mismatch count over the
    whole tensor."""
    import torch

    from oracle import qlinear_oracle as O

    out = {}
    cases = [("syl128_k3072", 3072, 128, "sylvester"), ("reg256_k3072", 3072, 256, "regular"),
             ("syl128_k12288", 12288, 128, "sylvester")]
    for name, K, g, kind in cases:
        x = gi.activation(1, 4096, K, "bf16")
        if kind == "sylvester":
            H = torch.tensor(scipy_hadamard(g), dtype=torch.float32) / (g ** 0.5)
        else:
            H = cr.build_hadamard(g, device="cpu", dtype=torch.float32)
        xr = cr.rotate_activation(torch.from_numpy(x).to(torch.bfloat16), H, group_size=g)
        q, s = i8.quantize_int8_axiswise(xr, dim=-1)
        q = q.numpy()
        s = s.numpy().reshape(-1)
        qo, so = O.quantize_int8_axiswise(O.rotate(x, g, kind, "bf16"), -1)
        diff = np.flatnonzero(q.reshape(-1) != qo.reshape(-1)).astype(np.int64)
        rot_ref = xr.contiguous().view(torch.int16).numpy().view(np.uint16).astype(np.int32)
        rot_orc = O.f32_to_bf16_bits(O.rotate(x, g, kind, "bf16")).astype(np.int32)
        out[f"{name}_q_sha"] = np.array(sha(q))
        out[f"{name}_s"] = s
        out[f"{name}_diff_pos"] = diff
        out[f"{name}_diff_val"] = q.reshape(-1)[diff]
        out[f"{name}_scale_rows_differ"] = np.array(int((s != so.reshape(-1)).sum()))
        out[f"{name}_rot_elems_differ"] = np.array(int((rot_ref != rot_orc).sum()))
        # largest difference in units of the bf16 spacing at the row's
        # absmax (values that nearly cancel differ by more ulps of their own)
        fr = xr.to(torch.float32).numpy()
        fo = O.rotate(x, g, kind, "bf16")
        amax = np.abs(fr).max(axis=1, keepdims=True)
        spacing = np.spacing(amax.astype(np.float32)) * 2.0 ** 16
        out[f"{name}_rot_max_diff_in_row_ulps"] = np.array(float((np.abs(fr - fo) / spacing).max()))
        print(name, "codes differing:", diff.size, "of", q.size, "scales differing:",
              int(out[f"{name}_scale_rows_differ"]), "rotated values differing:",
              int(out[f"{name}_rot_elems_differ"]), "largest difference in row-absmax ulps:",
              float(out[f"{name}_rot_max_diff_in_row_ulps"]))
    path = os.path.join(HERE, "golden_c1.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
