"""Loader nodes (``Load Diffusion Model Int8/Int4``, ``Int8 Pre-Lora
Loader``) and the LoRA model patchers, against stand-in ComfyUI modules.

CPU tests cover node registration, argument handling, the loader's class
flags, checkpoint metadata bridging and LoRA grouping; GPU tests check that
on-the-fly quantisation with a baked pre-LoRA and the patchers' bake-in
paths give the oracle's codes bit for bit."""
import json

import numpy as np
import pytest
import torch

import comfy_stubs as S
from conftest import cuda_ok
from oracle import qlinear_oracle as O

LAYERS = {"blocks.0.qkv": (384, 256), "blocks.0.proj": (256, 256), "img_in": (128, 256)}


@pytest.fixture(scope="module")
def C():
    return S.load_package_with_comfy()


def cq(d):
    return torch.tensor(list(json.dumps(d).encode("utf-8")), dtype=torch.uint8)


def float_weights(seed):
    rng = np.random.default_rng(seed)
    return {name: O.rnd("bf16", rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02))
            for name, (n, k) in LAYERS.items()}


def int8_checkpoint(seed=0, convrot=False):
    sd, ref = {}, {}
    for name, w in float_weights(seed).items():
        q, s = O.quantize_weight_int8(w, 256 if convrot else 0, "regular")
        ref[name] = (q, s)
        sd[name + ".weight"] = torch.from_numpy(q)
        sd[name + ".weight_scale"] = torch.from_numpy(s)
        conf = {"format": "int8_tensorwise", "per_row": True}
        if convrot:
            conf.update(convrot=True, convrot_groupsize=256)
        sd[name + ".comfy_quant"] = cq(conf)
        sd[name + ".bias"] = torch.zeros(w.shape[0])
    return sd, ref


def float_checkpoint(seed=0):
    ws = float_weights(seed)
    sd = {name + ".weight": torch.from_numpy(w).to(torch.bfloat16) for name, w in ws.items()}
    return sd, ws


def test_node_mappings(C):
    m = C.NODE_CLASS_MAPPINGS
    assert set(m) == {"OTUNetLoaderW8A8", "INT8PreLoraLoader", "UNetLoaderINT4ConvRot"}
    assert C.NODE_DISPLAY_NAME_MAPPINGS["OTUNetLoaderW8A8"] == "Load Diffusion Model Int8"
    S.register_file("diffusion_models", "listed.safetensors", {})
    it = m["OTUNetLoaderW8A8"].INPUT_TYPES()["required"]
    assert "listed.safetensors" in it["unet_name"][0]
    assert it["lora_mode"][0] == ["None", "Stochastic", "Dynamic"]
    assert m["UNetLoaderINT4ConvRot"].INPUT_TYPES()["required"]["convrot_groupsize"][1]["default"] == 256
    assert m["OTUNetLoaderW8A8"].RETURN_TYPES == ("MODEL",)


def test_int8_loader_prequantized(C):
    sd, _ = int8_checkpoint(1)
    S.register_file("diffusion_models", "int8.safetensors", sd, {"format": "int8"})
    Ops = C.int8_quant.Int8TensorwiseOps
    (model,) = C.int8_unet_loader.UNetLoaderINTW8A8().load_unet("int8.safetensors", "bf16", "flux2", False,
                                                                  enable_convrot=False)
    assert isinstance(model, C.int8_quant.INT8ModelPatcher)
    for name in LAYERS:
        lin = S.get_attr(model.model, name)
        assert lin._is_quantized and lin._is_per_row and lin.weight.dtype == torch.int8
    assert Ops.excluded_names == C.int8_unet_loader.INT8_MODEL_TYPE_EXCLUSIONS["flux2"]
    assert Ops.compute_dtype == torch.bfloat16 and Ops._is_prequantized
    assert Ops.lora_patches == {} and not hasattr(Ops, "applied_lora_patches")
    factory, args = model.cached_patcher_init
    assert factory is C.int8_unet_loader._load_int8_unet_cached_patcher and args[0] == "int8.safetensors"
    assert model.model._int8_source_metadata == {"format": "int8"}


def test_int8_loader_lora_mode_arguments(C):
    sd, _ = int8_checkpoint(2)
    S.register_file("diffusion_models", "int8b.safetensors", sd)
    Ops = C.int8_quant.Int8TensorwiseOps
    node = C.int8_unet_loader.UNetLoaderINTW8A8()
    node.load_unet("int8b.safetensors", "default", "wan", False, lora_mode=True)
    assert Ops.lora_mode == "Dynamic" and Ops.dynamic_lora and Ops.compute_dtype is None
    node.load_unet("int8b.safetensors", "fp16", "wan", False, lora_mode="bogus")
    assert Ops.lora_mode == "None" and not Ops.dynamic_lora and Ops.compute_dtype == torch.float16
    Ops.dynamic_lora = False


def test_pre_lora_loader_reads_dynamic_inputs(C):
    node = C.int8_unet_loader.PreLoraLoader()
    prompt = {"7": {"inputs": {"lora_name_1": "a.safetensors", "lora_strength_1": 0.756,
                               "lora_name_2": "None", "lora_strength_2": 1.0,
                               "lora_name_3": "b.safetensors", "lora_strength_3": 0.0,
                               "lora_name_4": "c.safetensors", "lora_strength_4": -1.0}}}
    (loras,) = node.load_pre_lora(prompt=prompt, id="7")
    assert loras == [{"lora_name": "a.safetensors", "lora_strength": 0.76},
                     {"lora_name": "c.safetensors", "lora_strength": -1.0}]
    (loras,) = node.load_pre_lora(lora_name="d.safetensors", lora_strength=0.5)
    assert loras == [{"lora_name": "d.safetensors", "lora_strength": 0.5}]


def test_group_pre_loras_normalizes_keys(C):
    d1 = torch.ones(384, 256)
    d2 = torch.ones(64, 256)
    S.register_file("loras", "l1.safetensors", {"diffusion_model.blocks.0.qkv.weight": d1,
                                                ("transformer.img_in.weight", (0, 0, 64)): d2})
    Ops = C.int8_quant.Int8TensorwiseOps
    g = C.loader_common.group_pre_loras(Ops, {}, {}, [{"lora_name": "l1.safetensors", "lora_strength": 0.5},
                                                      {"lora_name": "None", "lora_strength": 1.0}])
    assert set(g) == {"blocks.0.qkv.weight", "img_in.weight"}
    v, offset, function, strength = g["img_in.weight"][0]
    assert v is d2 and offset == (0, 0, 64) and function is None and strength == 0.5
    assert not Ops.skeleton_meta_init


def test_int4_metadata_bridge(C):
    sd = {"model.diffusion_model.blocks.0.qkv.weight": torch.zeros(384, 128, dtype=torch.int8),
          "img_in.weight": torch.zeros(128, 128, dtype=torch.int8)}
    layers = {"blocks.0.qkv": {"format": "convrot_w4a4", "convrot_groupsize": 256},
              "img_in": {"format": "convrot_w4a4", "convrot_groupsize": 128},
              "missing": {"format": "convrot_w4a4"},
              "other": {"format": "int8_tensorwise"}}
    n = C.int4_unet_loader.bridge_convrot_w4a4_metadata(sd, {"_quantization_metadata": json.dumps({"layers": layers})})
    assert n == 2
    conf = json.loads(bytes(sd["model.diffusion_model.blocks.0.qkv.comfy_quant"].tolist()).decode())
    assert conf == {"format": "convrot_w4a4", "convrot_groupsize": 256}
    assert "img_in.comfy_quant" in sd
    assert C.int4_unet_loader.bridge_convrot_w4a4_metadata({}, None) == 0


def test_int8_prequantized_pre_lora_is_reported_unmatched(C, caplog):
    sd, _ = int8_checkpoint(3)
    S.register_file("diffusion_models", "int8c.safetensors", sd)
    S.register_file("loras", "l2.safetensors", {"blocks.0.proj.weight": torch.ones(256, 256)})
    with caplog.at_level("WARNING"):
        C.int8_unet_loader.UNetLoaderINTW8A8().load_unet(
            "int8c.safetensors", "default", "flux2", False,
            pre_lora=[{"lora_name": "l2.safetensors", "lora_strength": 1.0}])
    assert "NOT matched" in caplog.text  # int8 weights are not re-baked at load


gpu = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_int8_loader_otf_with_pre_lora(C):
    sd, ws = float_checkpoint(4)
    delta = (np.random.default_rng(5).standard_normal((384, 256)) * 0.01).astype(np.float32)
    S.register_file("diffusion_models", "bf16.safetensors", sd)
    S.register_file("loras", "l3.safetensors", {"diffusion_model.blocks.0.qkv.weight": torch.from_numpy(delta)})
    (model,) = C.int8_unet_loader.UNetLoaderINTW8A8().load_unet(
        "bf16.safetensors", "bf16", "flux2", True, enable_convrot=True,
        pre_lora=[{"lora_name": "l3.safetensors", "lora_strength": 0.5}])
    qkv = model.model.blocks[0].qkv
    assert qkv._is_quantized and qkv._use_convrot
    # bake in float32 (the stand-in LoRA compute dtype), back to bf16, then
    # float32 -> ConvRot -> per-row int8
    patched = O.rnd("bf16", ws["blocks.0.qkv"] + np.float32(0.5) * delta)
    q, s = O.quantize_weight_int8(patched, 256, "regular")
    np.testing.assert_array_equal(qkv.weight.numpy(), q)
    np.testing.assert_array_equal(qkv.weight_scale.numpy(), s)
    proj = model.model.blocks[0].proj
    q2, s2 = O.quantize_weight_int8(ws["blocks.0.proj"], 256, "regular")
    np.testing.assert_array_equal(proj.weight.numpy(), q2)
    assert not model.model.img_in._is_quantized  # excluded for flux2


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
@pytest.mark.parametrize("convrot", [False, True])
def test_int8_patcher_bake_matches_oracle(C, convrot):
    sd, ref = int8_checkpoint(6, convrot)
    S.register_file("diffusion_models", f"int8d{convrot}.safetensors", sd)
    Ops = C.int8_quant.Int8TensorwiseOps
    (model,) = C.int8_unet_loader.UNetLoaderINTW8A8().load_unet(f"int8d{convrot}.safetensors", "bf16", "flux2",
                                                                  False, lora_mode="None")
    delta = (np.random.default_rng(7).standard_normal((256, 256)) * 0.01).astype(np.float32)
    key = "blocks.0.proj.weight"
    model.add_patches({key: torch.from_numpy(delta)}, 0.75)
    out = model.patch_weight_to_device(key, device_to=torch.device("cuda"), return_weight=True)
    q, s = ref["blocks.0.proj"]
    g = 256 if convrot else 0
    w = O.dequant_unrotate_int8(q, s, g, "regular") + np.float32(0.75) * delta
    np.testing.assert_array_equal(out.cpu().numpy(), O.rotate_requant_int8(w, s, g, "regular"))
    # a second bake starts again from the backed-up base weight
    model.patch_weight_to_device(key, device_to=torch.device("cuda"))
    out2 = model.patch_weight_to_device(key, device_to=torch.device("cuda"), return_weight=True)
    np.testing.assert_array_equal(out2.cpu().numpy(), out.cpu().numpy())
    # the low-VRAM callable gives the same codes
    lin = model.model.blocks[0].proj
    lv = C.int8_quant.INT8LowVramPatch(key, model.patches, lin, "None")
    np.testing.assert_array_equal(lv(torch.from_numpy(q).cuda()).cpu().numpy(), out.cpu().numpy())
    Ops.lora_mode = "None"


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_int8_patcher_dynamic_lora_forward(C):
    sd, ref = int8_checkpoint(8, convrot=True)
    S.register_file("diffusion_models", "int8e.safetensors", sd)
    Ops = C.int8_quant.Int8TensorwiseOps
    (model,) = C.int8_unet_loader.UNetLoaderINTW8A8().load_unet("int8e.safetensors", "bf16", "flux2", False,
                                                                  enable_convrot=True, lora_mode="Dynamic")
    try:
        rng = np.random.default_rng(9)
        up = torch.from_numpy(rng.standard_normal((256, 8)).astype(np.float32) * 0.05)
        down = torch.from_numpy(rng.standard_normal((8, 256)).astype(np.float32) * 0.05)
        key = "blocks.0.proj.weight"
        model.add_patches({key: S.LoraAdapter(up, down, alpha=4.0)}, 1.0)
        model.patch_weight_to_device(key)
        lin = model.model.blocks[0].proj
        assert len(lin.lora_patches) == 1
        x = torch.randn(64, 256, device="cuda", dtype=torch.bfloat16)
        y = lin(x)
        lin_patches, lin.lora_patches = lin.lora_patches, []
        y0 = lin(x)
        lin.lora_patches = lin_patches
        # the low-rank branch in the unrotated basis: x @ (0.5 * up @ down)^T
        want = (x.float() @ (0.5 * up @ down).T.cuda()).cpu()
        got = (y.float() - y0.float()).cpu()
        assert torch.allclose(got, want, atol=2e-2, rtol=2e-2)
    finally:
        Ops.dynamic_lora = False
        Ops.lora_mode = "None"


def int4_checkpoint(seed=10):
    sd, ref = {}, {}
    for name, w in float_weights(seed).items():
        wr = O.rotate(w, 256, "regular", "f32")
        q, s = O.quantize_signed_int4_rowwise(wr, "f32")
        ref[name] = (q, s)
        sd[name + ".weight"] = torch.from_numpy(O.pack_int4_row_major(q))
        sd[name + ".weight_scale"] = torch.from_numpy(s)
        sd[name + ".comfy_quant"] = cq({"format": "convrot_w4a4", "convrot_groupsize": 256})
    return sd, ref


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_int4_loader_and_patcher_bake(C):
    sd, ref = int4_checkpoint()
    S.register_file("diffusion_models", "int4.safetensors", sd)
    (model,) = C.int4_unet_loader.UNetLoaderINT4ConvRot().load_unet("int4.safetensors", "flux2", False)
    assert isinstance(model, C.int4_quant.Int4ModelPatcher)
    lin = model.model.blocks[0].proj
    assert lin._is_quantized and lin._linear_dtype == "int4"
    delta = (np.random.default_rng(11).standard_normal((256, 256)) * 0.01).astype(np.float32)
    key = "blocks.0.proj.weight"
    model.add_patches({key: torch.from_numpy(delta)}, 1.0)
    out = model.patch_weight_to_device(key, return_weight=True)
    q, s = ref["blocks.0.proj"]
    w = O.rotate(q.astype(np.float32) * s.reshape(-1, 1), 256, "regular", "f32") + delta
    wr = O.rotate(w, 256, "regular", "f32")
    want = np.clip(np.rint(wr / s.reshape(-1, 1)), -7, 7).astype(np.int8)
    np.testing.assert_array_equal(out.cpu().numpy(), O.pack_int4_row_major(want))
