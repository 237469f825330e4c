"""On-disk round trip of quantised models: load -> save -> load restores
every quantised layer bit for bit (weights, scales, bias, ConvRot and
per-row flags), through a safetensors file, in the formats the reference's
save node writes (int8_save.py:219-256) and its loaders read."""
import json

import numpy as np
import torch
from torch import nn

import golden_inputs as gi
from comfy_stubs import load_package_with_comfy
from oracle import qlinear_oracle as O

import pytest


@pytest.fixture(scope="module")
def C():
    return load_package_with_comfy()


def cq(d):
    return torch.tensor(list(json.dumps(d).encode()), dtype=torch.uint8)


def _int8_model(C):
    Ops = C.Int8TensorwiseOps
    m = nn.Module()
    m.per_row = Ops.Linear(512, 96)
    m.tensorwise = Ops.Linear(256, 64, bias=False)
    m.plain = Ops.Linear(32, 16)
    wq, ws = O.quantize_weight_int8(gi.weight(61, 96, 512), 128, "sylvester")
    sd = {"per_row.weight": torch.from_numpy(wq), "per_row.weight_scale": torch.from_numpy(ws),
          "per_row.bias": torch.from_numpy(gi.bias(61, 96, "bf16")).to(torch.bfloat16),
          "per_row.comfy_quant": cq({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 128,
                                     "per_row": True}),
          "tensorwise.weight": torch.from_numpy(gi.int8_weight(62, 64, 256)), "tensorwise.weight_scale": torch.tensor(0.01),
          "plain.weight": torch.from_numpy(gi.weight(63, 16, 32)).to(torch.bfloat16),
          "plain.bias": torch.zeros(16, dtype=torch.bfloat16)}
    return m, sd


def _load(m, sd):
    missing, unexpected = [], []
    for name, mod in m.named_children():
        errs = []
        mod._load_from_state_dict(sd, name + ".", {}, True, missing, unexpected, errs)
        assert not errs
    assert not missing
    return m


def _same_layers(a, b):
    for (na, ma), (nb, mb) in zip(a.named_children(), b.named_children()):
        assert na == nb
        for attr in ("_is_quantized", "_is_per_row", "_use_convrot", "_convrot_groupsize"):
            assert getattr(ma, attr, None) == getattr(mb, attr, None), (na, attr)
        for t in ("weight", "weight_scale", "bias"):
            x, y = getattr(ma, t, None), getattr(mb, t, None)
            assert (x is None) == (y is None), (na, t)
            if x is not None:
                assert x.dtype == y.dtype and torch.equal(x.reshape(-1), y.reshape(-1)), (na, t)


def test_int8_round_trip_through_safetensors(C, tmp_path):
    Ops = C.Int8TensorwiseOps
    saved_convrot = Ops.enable_convrot
    try:
        src, sd = _int8_model(C)
        _load(src, dict(sd))
        assert src.per_row._is_per_row and src.per_row._use_convrot and not src.tensorwise._is_per_row
        path = str(tmp_path / "model.safetensors")
        out = C.int8_save.save_quantized(src, path)
        conf = json.loads(bytes(out["per_row.comfy_quant"].tolist()))
        assert conf == {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 128, "per_row": True}
        assert json.loads(bytes(out["tensorwise.comfy_quant"].tolist())) == \
            {"format": "int8_tensorwise", "convrot": False, "per_row": False}
        assert "plain.comfy_quant" not in out and out["plain.weight"].dtype == torch.bfloat16
        from safetensors.torch import load_file
        dst, _ = _int8_model(C)
        _load(dst, load_file(path))
        _same_layers(src, dst)
    finally:
        Ops.enable_convrot = saved_convrot


def test_int4_round_trip(C, golden):
    Ops = C.Int4ConvRotOps
    m = nn.Module()
    m.w4a4 = Ops.Linear(512, 128)
    m.mixed = Ops.Linear(256, 64)
    sd = {"w4a4.weight": torch.from_numpy(golden["i4w_packed"]), "w4a4.weight_scale": torch.from_numpy(golden["i4w_scale"]),
          "w4a4.bias": torch.from_numpy(gi.bias(9, 128, "bf16")).to(torch.bfloat16),
          "w4a4.comfy_quant": cq({"format": "convrot_w4a4", "convrot_groupsize": 256}),
          "mixed.weight": torch.from_numpy(gi.int8_weight(64, 64, 256)), "mixed.weight_scale": torch.rand(64, 1),
          "mixed.bias": torch.zeros(64, dtype=torch.bfloat16),
          "mixed.comfy_quant": cq({"format": "int8_tensorwise", "per_row": True})}
    _load(m, dict(sd))
    out = C.int8_save.quantized_state_dict(m, prefix="model.diffusion_model.")
    assert json.loads(bytes(out["model.diffusion_model.w4a4.comfy_quant"].tolist())) == \
        {"format": "convrot_w4a4", "convrot_groupsize": 256, "linear_dtype": "int4"}
    back = nn.Module()
    back.w4a4 = Ops.Linear(512, 128)
    back.mixed = Ops.Linear(256, 64)
    stripped = {k[len("model.diffusion_model."):]: v for k, v in out.items()}
    _load(back, stripped)
    _same_layers(m, back)
    np.testing.assert_array_equal(back.w4a4.weight.numpy(), golden["i4w_packed"])
