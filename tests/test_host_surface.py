"""The ComfyUI operator surface (custom operations, weight formats, layout
registration) with stub ComfyUI modules.  CPU-only parts here; the GPU
forward parity of the same classes is in the gpu-marked tests below."""
import json

import numpy as np
import pytest
import torch

import golden_inputs as gi
from comfy_stubs import load_package_with_comfy
from conftest import cuda_ok
from oracle import qlinear_oracle as O


@pytest.fixture(scope="module")
def C():
    return load_package_with_comfy()


def cq(d):
    return torch.tensor(list(json.dumps(d).encode()), dtype=torch.uint8)


def test_classes_defined_and_layout_registered(C):
    import sys
    assert C.Int8TensorwiseOps is not None and C.Int4ConvRotOps is not None
    qo = sys.modules["comfy.quant_ops"]
    assert "int8_tensorwise" in qo.QUANT_ALGOS
    assert qo.QUANT_ALGOS["int8_tensorwise"]["parameters"] == {"weight_scale", "input_scale"}
    assert "Int8TensorwiseLayout" in qo.LAYOUTS
    L = qo.LAYOUTS["Int8TensorwiseLayout"]
    p = L.Params(scale=torch.tensor(0.5))
    assert L.dequantize(torch.tensor([2], dtype=torch.int8), p).item() == 1.0
    assert set(L.state_dict_tensors(torch.zeros(1), p)) == {"", "weight_scale"}


def test_int8_prequantized_per_row_load(C):
    Ops = C.Int8TensorwiseOps
    lin = Ops.Linear(256, 64)
    sd = {"blk.weight": torch.zeros(64, 256, dtype=torch.int8), "blk.weight_scale": torch.ones(64, 1),
          "blk.bias": torch.zeros(64, dtype=torch.bfloat16),
          "blk.comfy_quant": cq({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 128,
                                 "per_row": True}),
          "blk.input_scale": torch.ones(())}
    missing, unexpected, errs = [], [], []
    lin._load_from_state_dict(sd, "blk.", {}, True, missing, unexpected, errs)
    assert lin._is_quantized and lin._is_per_row and lin._use_convrot and lin._convrot_groupsize == 128
    assert lin.weight.dtype == torch.int8 and lin.weight_scale.shape == (64, 1)
    assert not sd and not missing and not errs
    assert C.int8_quant.rot_for_group(128) == ("sylvester", 128)
    assert C.int8_quant.rot_for_group(256) == ("regular", 256)


def test_int8_scalar_scale_and_prefix_variants(C):
    lin = C.Int8TensorwiseOps.Linear(64, 32, bias=False)
    sd = {"model.x.weight_scale": torch.tensor(0.25), "x.weight": torch.zeros(32, 64, dtype=torch.int8)}
    lin._load_from_state_dict(sd, "x.", {}, True, [], [], [])
    assert lin._is_quantized and not lin._is_per_row
    assert lin.weight_scale.shape == (1,) and float(lin.weight_scale) == 0.25


def test_int8_high_precision_not_quantized_without_otf(C):
    Ops = C.Int8TensorwiseOps
    Ops.dynamic_quantize = False
    lin = Ops.Linear(64, 32)
    sd = {"l.weight": torch.randn(32, 64, dtype=torch.bfloat16), "l.bias": torch.zeros(32, dtype=torch.bfloat16)}
    lin._load_from_state_dict(sd, "l.", {}, True, [], [], [])
    assert not lin._is_quantized and lin.weight.dtype == torch.bfloat16


def test_int8_missing_weight_reported(C):
    lin = C.Int8TensorwiseOps.Linear(64, 32)
    missing = []
    lin._load_from_state_dict({}, "m.", {}, True, missing, [], [])
    assert missing == ["m.weight"]


def test_w4a8_format_load(C):
    lin = C.Int8TensorwiseOps.Linear(256, 96)
    packed, cb, sch, srel = gi.asym_w4a8(10, 96, 256, 16)
    sd = {"w.weight": torch.from_numpy(packed), "w.weight_codebook": torch.from_numpy(cb),
          "w.weight_s_channel": torch.from_numpy(sch), "w.weight_s_rel": torch.from_numpy(srel),
          "w.comfy_quant": cq({"format": "asym_w4a8_int8", "group_size": 16})}
    lin._load_from_state_dict(sd, "w.", {}, True, [], [], [])
    assert lin._is_w4a8 and lin._w4a8_group_size == 16 and lin._is_per_row
    assert lin.weight.shape == (96, 128)


def test_int4_formats_load(C):
    Ops = C.Int4ConvRotOps
    lin = Ops.Linear(512, 128)
    sd = {"a.weight": torch.zeros(128, 256, dtype=torch.int8), "a.weight_scale": torch.ones(128),
          "a.comfy_quant": cq({"format": "convrot_w4a4", "convrot_groupsize": 256})}
    errs = []
    lin._load_from_state_dict(sd, "a.", {}, True, [], [], errs)
    assert lin._is_quantized and lin._linear_dtype == "int4" and not errs
    lin2 = Ops.Linear(512, 128)
    sd = {"b.weight": torch.zeros(128, 512, dtype=torch.int8), "b.weight_scale": torch.ones(128, 1),
          "b.comfy_quant": cq({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256})}
    lin2._load_from_state_dict(sd, "b.", {}, True, [], [], [])
    assert lin2._linear_dtype == "int8_tensorwise" and lin2._use_convrot and lin2._is_per_row
    lin3 = Ops.Linear(256, 64)
    errs = []
    sd = {"c.weight": torch.zeros(64, 100, dtype=torch.int8), "c.weight_scale": torch.ones(64),
          "c.comfy_quant": cq({"format": "convrot_w4a4"})}
    lin3._load_from_state_dict(sd, "c.", {}, True, [], [], errs)
    assert errs and "in_features" in errs[0]


def test_w4a8_metadata_bridge(C):
    sd = {"model.diffusion_model.blk.attn.weight": torch.zeros(1)}
    meta = {"_quantization_metadata": json.dumps({"layers": {"blk.attn": {"format": "asym_w4a8_int8", "group_size": 16},
                                                             "other": {"format": "int8_tensorwise"}}})}
    n = C.w4a8_int8.bridge_w4a8_metadata_to_comfy_quant(sd, meta)
    assert n == 1
    conf = json.loads(bytes(sd["model.diffusion_model.blk.attn.comfy_quant"].tolist()))
    assert conf == {"format": "asym_w4a8_int8", "group_size": 16}
    assert C.w4a8_int8.bridge_w4a8_metadata_to_comfy_quant({}, None) == 0


def test_pack_unpack_torch_matches_oracle(C, golden):
    nib = torch.from_numpy(gi.nibbles(7, 64, 128))
    p = C.int4_quant.pack_int4_row_major(nib)
    np.testing.assert_array_equal(p.numpy(), golden["i4_pack"])
    np.testing.assert_array_equal(C.int4_quant.unpack_int4_row_major(p).numpy(), nib.numpy())


def test_build_hadamard_matches_reference(C, golden):
    for g in (16, 64, 256):
        H = C.convrot.build_hadamard(g)
        np.testing.assert_array_equal(H.numpy(), golden[f"rot_reg{g}_H"])
        assert C.convrot.hadamard_kind(H) == "regular"
    with pytest.raises(ValueError):
        C.convrot.build_hadamard(128)
    Hs = C.convrot.build_hadamard(128, kind="sylvester")
    np.testing.assert_array_equal(Hs.numpy(), golden["rot_syl128_H"])
    # an untagged matrix is identified by its sign pattern
    assert C.convrot.hadamard_kind(torch.from_numpy(golden["rot_syl128_H"])) == "sylvester"


def test_torch_cpu_path_matches_oracle():
    """The CPU baseline (the reference's torch CPU calls) agrees with the
    numpy oracle: bit-exact without rotation."""
    from oracle import torch_cpu_path as R
    x = gi.activation(30, 64, 512, "bf16")
    w = gi.weight(30, 96, 512)
    b = gi.bias(30, 96, "bf16")
    wq, ws = R.quantize_int8_axiswise(torch.from_numpy(w), dim=1)
    y = R.convrot_w8a8_linear(torch.from_numpy(x).to(torch.bfloat16), None, 0, wq, ws,
                              torch.from_numpy(b).to(torch.bfloat16), torch.bfloat16)
    yo = O.int8_forward_dynamic_per_row(x, wq.numpy(), ws.numpy(), b, "bf16")
    np.testing.assert_array_equal(y.float().numpy(), yo)


# --------------------------------------------------------------------------
# GPU forward of the operator classes
# --------------------------------------------------------------------------

gpu = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_int8_linear_forward_otf_convrot(C):
    Ops = C.Int8TensorwiseOps
    Ops.dynamic_quantize, Ops.enable_convrot, Ops.excluded_names = True, True, []
    Ops.compute_dtype = None
    lin = Ops.Linear(512, 256)
    w = gi.weight(31, 256, 512)
    b = gi.bias(31, 256, "bf16")
    sd = {"l.weight": torch.from_numpy(w).to(torch.bfloat16), "l.bias": torch.from_numpy(b).to(torch.bfloat16)}
    lin._load_from_state_dict(sd, "l.", {}, True, [], [], [])
    assert lin._is_quantized and lin._use_convrot
    x = gi.activation(31, 2 * 24, 512, "bf16")
    y = lin(torch.from_numpy(x).reshape(2, 24, 512).to(torch.bfloat16).cuda())
    assert y.shape == (2, 24, 256)
    wq, ws = O.quantize_weight_int8(O.rnd("bf16", w), 256, "regular")
    yo = O.int8_forward_dynamic_per_row(O.rotate(x, 256, "regular", "bf16"), wq, ws, b, "bf16")
    np.testing.assert_array_equal(y.reshape(48, 256).float().cpu().numpy(), yo)
    Ops.dynamic_quantize, Ops.enable_convrot = False, False


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_int8_linear_forward_w4a8_cached(C, golden):
    lin = C.Int8TensorwiseOps.Linear(256, 96)
    packed, cb, sch, srel = gi.asym_w4a8(10, 96, 256, 16)
    sd = {"w.weight": torch.from_numpy(packed), "w.weight_codebook": torch.from_numpy(cb),
          "w.weight_s_channel": torch.from_numpy(sch), "w.weight_s_rel": torch.from_numpy(srel),
          "w.comfy_quant": cq({"format": "asym_w4a8_int8", "group_size": 16})}
    lin._load_from_state_dict(sd, "w.", {}, True, [], [], [])
    lin.cuda()
    x = gi.activation(32, 33, 256, "bf16")
    y = lin(torch.from_numpy(x).to(torch.bfloat16).cuda())
    yo = O.int8_forward_dynamic_per_row(x, golden["w4a8_q"], golden["w4a8_s"], None, "bf16")
    np.testing.assert_array_equal(y.float().cpu().numpy(), yo)
    assert len(lin._w4a8_cache) == 1


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_int4_linear_forward(C, golden):
    lin = C.Int4ConvRotOps.Linear(512, 128)
    sd = {"a.weight": torch.from_numpy(golden["i4w_packed"]), "a.weight_scale": torch.from_numpy(golden["i4w_scale"]),
          "a.bias": torch.from_numpy(gi.bias(9, 128, "bf16")).to(torch.bfloat16),
          "a.comfy_quant": cq({"format": "convrot_w4a4", "convrot_groupsize": 256})}
    lin._load_from_state_dict(sd, "a.", {}, True, [], [], [])
    x = gi.activation(9, 37, 512, "bf16")
    y = lin(torch.from_numpy(x).to(torch.bfloat16).cuda())
    got = y.cpu().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, golden["i4fwd_y"])


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
@pytest.mark.parametrize("convrot", [False, True])
def test_int8_linear_dynamic_lora_fused_add(C, convrot):
    """One full-width dynamic LoRA runs its add in the GEMM epilogue: equal
    to the eager ``y + lora_y.to(y.dtype)`` (int8_quant.py:718-729); a
    sliced patch (split qkv) and two patches keep the eager form and agree
    with it too."""
    Ops = C.Int8TensorwiseOps
    Ops.dynamic_quantize, Ops.enable_convrot, Ops.excluded_names = True, convrot, []
    Ops.compute_dtype = None
    K, N, r = 512, 384, 16
    lin = Ops.Linear(K, N)
    w = gi.weight(41, N, K)
    b = gi.bias(41, N, "bf16")
    sd = {"l.weight": torch.from_numpy(w).to(torch.bfloat16), "l.bias": torch.from_numpy(b).to(torch.bfloat16)}
    lin._load_from_state_dict(sd, "l.", {}, True, [], [], [])
    x = torch.from_numpy(gi.activation(41, 2 * 40, K, "bf16")).reshape(2, 40, K).to(torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(3)
    lD = (torch.randn((r, K), generator=g) * 0.05).to(torch.bfloat16)
    lU = (torch.randn((N, r), generator=g) * 0.05).to(torch.bfloat16)
    lU2 = (torch.randn((128, r), generator=g) * 0.05).to(torch.bfloat16)
    lin.lora_patches = []
    y0 = lin(x).reshape(-1, N)
    x2 = x.reshape(-1, K)
    xl = C.ops.rotate(x2, *C.int8_quant.rot_for_group(256)) if convrot else x2

    def up(d, u):
        return torch.nn.functional.linear(torch.nn.functional.linear(xl, d.cuda()), u.cuda()).to(torch.bfloat16)

    lin.lora_patches = [(lD, lU, None, None)]
    assert torch.equal(lin(x).reshape(-1, N), y0 + up(lD, lU))
    lin.lora_patches = [(lD, lU2, 128, 128)]
    ref = y0.clone()
    ref[:, 128:256] = ref[:, 128:256] + up(lD, lU2)
    assert torch.equal(lin(x).reshape(-1, N), ref)
    lin.lora_patches = [(lD, lU, None, None), (lD, lU, None, None)]
    assert torch.equal(lin(x).reshape(-1, N), (y0 + up(lD, lU)) + up(lD, lU))
    lin.lora_patches = []
    Ops.dynamic_quantize, Ops.enable_convrot = False, False
