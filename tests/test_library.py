"""The kernels as torch.library custom operators (namespace qlin_b200).

CPU: every operator is registered with a fake implementation whose output
shapes and dtypes are those of the eager entry points (checked under
FakeTensorMode on fake CUDA tensors, no GPU needed), and a CPU tensor finds
no kernel.  GPU: torch.library.opcheck on the activation and GEMM operators,
and torch.compile(fullgraph=True) over the quantised Linear modules and the
kitchen op, bit-equal to eager -- the reference advertises torch.compile
(README.md:19) and registers its kitchen op as a custom op
(rocm_int8_kitchen_patch.py:19-21).
"""
import json

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import golden_inputs as gi
from comfy_stubs import load_package_with_comfy
from conftest import cuda_ok

OPS = ["quant_act_int8", "quant_act_int8_norm", "quant_act_int8_cat", "quant_act_int8_situ", "qk_norm_rope_",
       "quant_act_int4", "rotate", "situ", "gemm_w8a8", "gemm_w8a8_fused", "int_mm", "int4_mm", "gemm_w4a4",
       "gemm_w4_g128", "quant_weight_int8", "quant_weight_int4", "requant_asym_w4a8", "dequant_int8",
       "requant_int8"]


def test_every_kernel_is_a_registered_operator(pkg):
    ns = torch.ops.qlin_b200
    for name in OPS:
        op = getattr(ns, name).default
        assert op.namespace == "qlin_b200"
        assert torch._library.utils.has_fake_kernel(op), name


def test_fake_shapes(pkg):
    L = pkg.library
    d = "cuda"
    with FakeTensorMode():
        x = torch.empty(40, 512, dtype=torch.bfloat16, device=d)
        q, s = L.quant_act_int8(x, ("sylvester", 128))
        assert (q.shape, q.dtype, s.shape, s.dtype) == ((40, 512), torch.int8, (40, 1), torch.float32)
        q, s = L.quant_act_int8_norm(x, None, "layer", 1e-6, None, torch.empty(2, 512, dtype=torch.bfloat16,
                                                                                device=d))
        assert q.shape == (40, 512) and s.shape == (40, 1)
        q, s = L.quant_act_int8_cat(x, torch.empty(40, 256, dtype=torch.bfloat16, device=d))
        assert q.shape == (40, 768)
        q, s = L.quant_act_int8_situ(x)
        assert q.shape == (40, 256) and s.shape == (40, 1)
        q, s = L.quant_act_int4(x, ("regular", 256))
        assert q.shape == (40, 512) and s.shape == (40,)
        q, s = L.quant_act_int4(x, ("sylvester", 128), group=128)
        assert s.shape == (40, 4)
        assert L.rotate(x, "regular", 256).shape == (40, 512)
        assert L.situ(torch.empty(2, 7, 64, dtype=torch.bfloat16, device=d)).shape == (2, 7, 32)
        w = torch.empty(96, 512, dtype=torch.int8, device=d)
        ws = torch.empty(96, 1, device=d)
        a = torch.empty(40, 512, dtype=torch.int8, device=d)
        sa = torch.empty(40, 1, device=d)
        y = L.gemm_w8a8(a, sa, w, ws, None, torch.float16)
        assert (y.shape, y.dtype) == ((40, 96), torch.float16)
        y = L.gemm_w8a8_fused(a, sa, w, ws, None, torch.bfloat16, gelu_from=48,
                              residual=torch.empty(40, 96, dtype=torch.bfloat16, device=d))
        assert (y.shape, y.dtype) == ((40, 96), torch.bfloat16)
        assert L.int_mm(a, w).dtype == torch.int32
        wp = torch.empty(96, 256, dtype=torch.int8, device=d)
        assert L.int4_mm(a, wp).shape == (40, 96)
        assert L.gemm_w4a4(a, torch.empty(40, device=d), wp, torch.empty(96, device=d)).shape == (40, 96)
        assert L.gemm_w4_g128(a, torch.empty(40, device=d), wp, torch.empty(96, 4, device=d)).shape == (40, 96)
        wf = torch.empty(96, 512, device=d)
        q, s = L.quant_weight_int8(wf, ("regular", 256))
        assert q.shape == (96, 512) and s.shape == (96, 1)
        q, s = L.quant_weight_int4(wf, None, 128)
        assert q.shape == (96, 256) and s.shape == (96, 4)
        q, s = L.requant_asym_w4a8(wp, torch.empty(16, device=d), torch.empty(96, device=d),
                                   torch.empty(96, 32, dtype=torch.uint8, device=d), 16)
        assert q.shape == (96, 512) and s.shape == (96, 1)
        assert L.dequant_int8(w, ws).dtype == torch.float32
        assert L.requant_int8(wf, ws, stochastic=True, seed=2 ** 64 - 1).shape == (96, 512)
        qkv = torch.empty(2, 10, 3 * 2 * 64, dtype=torch.bfloat16, device=d)
        assert L.qk_norm_rope_(qkv, 2, 64) is qkv


def test_cpu_tensor_has_no_kernel(pkg):
    with pytest.raises((NotImplementedError, RuntimeError)):
        pkg.library.quant_act_int8(torch.zeros(4, 16, dtype=torch.bfloat16))


# ---------------------------------------------------------------------------
# GPU: opcheck and torch.compile
# ---------------------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_opcheck(pkg):
    ns = torch.ops.qlin_b200
    x = torch.from_numpy(gi.activation(50, 33, 512, "bf16")).to(torch.bfloat16).cuda()
    w = torch.from_numpy(gi.weight(50, 96, 512)).cuda()
    wq, ws = pkg.ops.quant_weight_int8(w, ("regular", 256))
    xq, xs = pkg.ops.quant_act_int8(x, ("regular", 256))
    b = torch.zeros(96, dtype=torch.bfloat16, device="cuda")
    utils = ("test_schema", "test_faketensor")
    torch.library.opcheck(ns.quant_act_int8.default, (x, "sylvester", 128), test_utils=utils)
    torch.library.opcheck(ns.gemm_w8a8.default, (xq, xs, wq, ws, b, torch.bfloat16, True), test_utils=utils)
    torch.library.opcheck(ns.gemm_w8a8_fused.default, (xq, xs, wq, ws, b, torch.bfloat16, True, 48, None, None, -1),
                          test_utils=utils)
    torch.library.opcheck(ns.quant_act_int4.default, (x, "regular", 256, 0), test_utils=utils)


def _cq(d):
    return torch.tensor(list(json.dumps(d).encode()), dtype=torch.uint8)


@pytest.fixture(scope="module")
def C():
    return load_package_with_comfy()


def _compiled_equal(mod, x):
    torch._dynamo.reset()
    y_eager = mod(x)
    y_comp = torch.compile(mod, fullgraph=True)(x)
    assert y_comp.shape == y_eager.shape and y_comp.dtype == y_eager.dtype
    assert torch.equal(y_comp, y_eager)


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
@pytest.mark.parametrize("convrot", [False, True])
def test_compile_int8_linear(C, convrot):
    Ops = C.Int8TensorwiseOps
    Ops.dynamic_quantize, Ops.enable_convrot, Ops.excluded_names = True, convrot, []
    Ops.compute_dtype = None
    try:
        lin = Ops.Linear(512, 256)
        sd = {"l.weight": torch.from_numpy(gi.weight(51, 256, 512)).to(torch.bfloat16),
              "l.bias": torch.from_numpy(gi.bias(51, 256, "bf16")).to(torch.bfloat16)}
        lin._load_from_state_dict(sd, "l.", {}, True, [], [], [])
        lin.cuda()
        x = torch.from_numpy(gi.activation(51, 2 * 24, 512, "bf16")).reshape(2, 24, 512).to(torch.bfloat16).cuda()
        _compiled_equal(lin, x)
    finally:
        Ops.dynamic_quantize, Ops.enable_convrot = False, False


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_compile_int4_linear(C, golden):
    lin = C.Int4ConvRotOps.Linear(512, 128)
    sd = {"a.weight": torch.from_numpy(golden["i4w_packed"]), "a.weight_scale": torch.from_numpy(golden["i4w_scale"]),
          "a.bias": torch.from_numpy(gi.bias(9, 128, "bf16")).to(torch.bfloat16),
          "a.comfy_quant": _cq({"format": "convrot_w4a4", "convrot_groupsize": 256})}
    lin._load_from_state_dict(sd, "a.", {}, True, [], [], [])
    lin.cuda()
    x = torch.from_numpy(gi.activation(9, 37, 512, "bf16")).to(torch.bfloat16).cuda()
    _compiled_equal(lin, x)


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_compile_kitchen_int8_linear(pkg):
    kp = pkg.kitchen_patch
    x = torch.from_numpy(gi.activation(52, 64, 1024, "bf16")).to(torch.bfloat16).cuda()
    w = torch.from_numpy(gi.weight(52, 384, 1024)).cuda()
    wq, ws = pkg.ops.quant_weight_int8(w, ("regular", 256))
    b = torch.from_numpy(gi.bias(52, 384, "bf16")).to(torch.bfloat16).cuda()
    res = torch.from_numpy(gi.activation(53, 64, 384, "bf16")).to(torch.bfloat16).cuda()

    def f(x):
        return kp.int8_linear(x, wq, ws, b, torch.bfloat16, convrot=True, convrot_groupsize=256,
                              residual=res, residual_scale=None)

    torch._dynamo.reset()
    assert torch.equal(torch.compile(f, fullgraph=True)(x), f(x))
