"""Pin the numpy oracle against golden vectors from the reference's own code.

Bit-exact where the reference's math is element-wise or integer; the
rotation (a float32 library matmul in the reference, whose accumulation order
is unspecified) is bounded to 1 unit in the last place of the output dtype.
"""
import hashlib

import numpy as np
import pytest

import golden_inputs as gi
from oracle import qlinear_oracle as O


def bits(dtype, v):
    v = np.asarray(v, np.float32)
    if dtype == "bf16":
        return O.f32_to_bf16_bits(v)
    if dtype == "f16":
        return v.astype(np.float16).view(np.uint16)
    return v.view(np.uint32)


def f_of(dtype, b):
    if dtype == "bf16":
        return O.bf16_bits_to_f32(b)
    return b.view(np.float16).astype(np.float32)


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_quantize_int8_axiswise(golden, dt):
    x = gi.activation(0, 37, 256, dt, zero_row=5)
    q, s = O.quantize_int8_axiswise(x, dim=-1)
    np.testing.assert_array_equal(q, golden[f"q8_{dt}_q"])
    np.testing.assert_array_equal(s.view(np.uint32), golden[f"q8_{dt}_s"].view(np.uint32))
    assert s[5, 0] == np.float32(1e-30) and not q[5].any()


def test_quantize_int8_configs0_scale(golden):
    x = gi.activation(0, 4096, 3072, "bf16")
    q, s = O.quantize_int8_axiswise(x, dim=-1)
    np.testing.assert_array_equal(q[:4], golden["q8_c0_q_rows"])
    np.testing.assert_array_equal(s, golden["q8_c0_s"])
    assert hashlib.sha256(q.tobytes()).hexdigest() == str(golden["q8_c0_q_sha"])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_w8a8_per_row_forward(golden, dt):
    x = gi.activation(1, 37, 256, dt)
    w = gi.weight(1, 512, 256)
    wq, ws = O.quantize_int8_axiswise(w, dim=1)
    np.testing.assert_array_equal(wq, golden[f"w8_{dt}_wq"])
    np.testing.assert_array_equal(ws, golden[f"w8_{dt}_ws"])
    b = gi.bias(1, 512, dt)
    y = O.int8_forward_dynamic_per_row(x, wq, ws, b, dt)
    np.testing.assert_array_equal(bits(dt, y), golden[f"w8_{dt}_y"])
    y0 = O.int8_forward_dynamic_per_row(x, wq, ws, None, dt)
    np.testing.assert_array_equal(bits(dt, y0), golden[f"w8_{dt}_y_nobias"])


def test_w8a8_per_row_medium_outliers(golden):
    x = gi.activation(2, 256, 3072, "bf16")
    w = gi.weight(2, 384, 3072)
    wq, ws = O.quantize_int8_axiswise(w, dim=1)
    assert hashlib.sha256(wq.tobytes()).hexdigest() == str(golden["w8m_wq_sha"])
    np.testing.assert_array_equal(ws, golden["w8m_ws"])
    y = O.int8_forward_dynamic_per_row(x, wq, ws, gi.bias(2, 384, "bf16"), "bf16")
    np.testing.assert_array_equal(bits("bf16", y), golden["w8m_y"])


def test_w8a8_tensorwise_forward(golden):
    x = gi.activation(3, 37, 256, "f16")
    wq = gi.int8_weight(3, 512, 256)
    y = O.int8_forward_dynamic(x, wq, np.float32(0.01), gi.bias(3, 512, "f16"), "f16")
    np.testing.assert_array_equal(bits("f16", y), golden["w8t_y"])


@pytest.mark.parametrize("g", [16, 64, 256])
def test_regular_hadamard_matrix(golden, g):
    H = O.hadamard_int(g, "regular").astype(np.float32) * np.float32(O.hadamard_scale(g, "f32"))
    np.testing.assert_array_equal(H, golden[f"rot_reg{g}_H"])


def test_sylvester_and_regular128(golden):
    H = O.hadamard_int(128, "sylvester").astype(np.float32) * np.float32(O.hadamard_scale(128, "f32"))
    np.testing.assert_array_equal(H, golden["rot_syl128_H"])
    # the reference's build_hadamard rejects 128 (not a power of 4)
    assert int(golden["regular128_raises"]) == 1
    with pytest.raises(ValueError):
        O.hadamard_int(128, "regular")


@pytest.mark.parametrize("name,g,kind", [("rot_reg16", 16, "regular"), ("rot_reg64", 64, "regular"),
                                         ("rot_reg256", 256, "regular"), ("rot_syl128", 128, "sylvester")])
def test_rotate_activation_within_one_ulp(golden, name, g, kind):
    x = gi.activation(4, 32, 1024, "bf16")
    y = O.rotate(x, g, kind, "bf16")
    ref = golden[f"{name}_y"]
    mine = bits("bf16", y).astype(np.int32)
    # bf16 bit patterns of same-sign values are monotone: diff == ulp distance
    d = np.abs(mine - ref.astype(np.int32))
    same_sign = (mine >> 15) == (ref.astype(np.int32) >> 15)
    assert same_sign[d > 0].all()
    assert d.max() <= 1, d.max()
    assert (d > 0).mean() < 2e-3, (d > 0).mean()


def test_rotate_weight_fp32(golden):
    w = gi.weight(5, 32, 512)
    y = O.rotate(w, 256, "regular", "f32")
    ref = golden["rotw_y"]
    # two float32 summation orders of 256 terms: both within a few ulp of max
    np.testing.assert_allclose(y, ref, rtol=0, atol=16 * np.spacing(np.abs(ref).max()))
    exact = (w.astype(np.float64).reshape(32, 2, 256) @ O.hadamard_int(256, "regular")).reshape(32, 512) / 16
    assert np.abs(y - exact).max() <= 16 * np.spacing(np.abs(ref).max())


def test_int4_rowwise_quant(golden):
    xr_ref = O.bf16_bits_to_f32(golden["i4_xrot"]).reshape(37, 512)
    q, s = O.quantize_signed_int4_rowwise(xr_ref, "bf16")
    np.testing.assert_array_equal(q, golden["i4_q"])
    np.testing.assert_array_equal(s, golden["i4_s"])
    x16 = gi.activation(6, 37, 512, "f16")
    q, s = O.quantize_signed_int4_rowwise(x16, "f16")
    np.testing.assert_array_equal(q, golden["i4_f16_q"])
    np.testing.assert_array_equal(s, golden["i4_f16_s"])


def test_int4_pack_unpack(golden):
    nib = gi.nibbles(7, 64, 128)
    p = O.pack_int4_row_major(nib)
    np.testing.assert_array_equal(p, golden["i4_pack"])
    np.testing.assert_array_equal(O.unpack_int4_row_major(p), golden["i4_unpack"])
    np.testing.assert_array_equal(O.unpack_int4_row_major(p), nib)


def test_int4_weight_quant_and_forward(golden):
    w = gi.weight(8, 128, 512)
    pw, ps = O.quantize_convrot_w4a4_weight(w, 256, "regular")
    ref_p = golden["i4w_packed"]
    # rotation is float32 in both; codes may differ only where the rotated
    # value sits within an ulp of a rounding boundary
    diff = O.unpack_int4_row_major(pw).astype(int) - O.unpack_int4_row_major(ref_p).astype(int)
    assert np.abs(diff).max() <= 1 and (diff != 0).mean() < 1e-3
    np.testing.assert_allclose(ps, golden["i4w_scale"], rtol=1e-6)
    # forward from the reference's own packed weight, bit-exact int32 and bf16
    x = gi.activation(9, 37, 512, "bf16")
    b = gi.bias(9, 128, "bf16")
    xr = O.rotate(x, 256, "regular", "bf16")
    qa, sa = O.quantize_signed_int4_rowwise(xr, "bf16")
    acc = O.int_mm(qa, O.unpack_int4_row_major(ref_p))
    # the reference rotated with its own matmul; compare the int32 product on
    # the rows whose rotated activations agree bit for bit
    same = (O.f32_to_bf16_bits(xr) == O.f32_to_bf16_bits(O.rotate(x, 256, "regular", "bf16"))).all(axis=1)
    assert same.all()
    y = O.w4a4_rowwise_epilogue(golden["i4fwd_acc"], sa, golden["i4w_scale"], b, "bf16")
    ok_rows = (acc == golden["i4fwd_acc"]).all(axis=1)
    assert ok_rows.mean() > 0.9
    np.testing.assert_array_equal(bits("bf16", y), golden["i4fwd_y"])


def test_asym_w4a8_dequant_requant(golden):
    packed, cb, sch, srel = gi.asym_w4a8(10, 96, 256, 16)
    deq = O.dequant_asym_w4a8_to_float(packed, cb, sch, srel, 16)
    np.testing.assert_array_equal(deq, golden["w4a8_deq"])
    q, s = O.requant_asym_w4a8(packed, cb, sch, srel, 16)
    np.testing.assert_array_equal(q, golden["w4a8_q"])
    np.testing.assert_array_equal(s, golden["w4a8_s"])


def test_otf_weight_quant(golden):
    w = gi.weight(11, 48, 512)
    q, s = O.quantize_weight_int8(w, 256, "regular")
    d = q.astype(int) - golden["otf_q"].astype(int)
    assert np.abs(d).max() <= 1 and (d != 0).mean() < 1e-3
    np.testing.assert_allclose(s, golden["otf_s"], rtol=1e-6)


def test_lora_bake_roundtrip(golden):
    oq, os_ = golden["otf_q"], golden["otf_s"]
    wf = O.dequant_unrotate_int8(oq, os_, 256, "regular")
    np.testing.assert_allclose(wf, golden["lora_unrot"], rtol=0, atol=1e-6)
    delta = gi.weight(12, 48, 512) * np.float32(0.05)
    q = O.rotate_requant_int8(golden["lora_unrot"] + delta, os_, 256, "regular")
    d = q.astype(int) - golden["lora_q"].astype(int)
    assert np.abs(d).max() <= 1 and (d != 0).mean() < 1e-3
    # with the reference's re-rotated weight as input the requant is bit-exact
    np.testing.assert_array_equal(O.quantize_int8(golden["lora_rerot"], os_), golden["lora_q"])


@pytest.mark.parametrize("name,K,g,kind", [("syl128_k3072", 3072, 128, "sylvester"),
                                           ("reg256_k3072", 3072, 256, "regular")])
def test_rotated_codes_vs_reference_full_size(golden_c1, name, K, g, kind):
    """The oracle's rotate + quantise at the ConvRot linear's full size
    (4096 tokens) against the reference's codes: they differ exactly at the
    positions the golden file lists (13 of 12.6 M codes for Sylvester 128,
    none for regular 256) and the per-token scales are equal."""
    import hashlib
    x = gi.activation(1, 4096, K, "bf16")
    q, s = O.quantize_int8_axiswise(O.rotate(x, g, kind, "bf16"), -1)
    qf = q.reshape(-1).copy()
    pos = golden_c1[f"{name}_diff_pos"]
    assert (qf[pos] != golden_c1[f"{name}_diff_val"]).all()
    qf[pos] = golden_c1[f"{name}_diff_val"]
    assert hashlib.sha256(qf.tobytes()).hexdigest() == str(golden_c1[f"{name}_q_sha"])
    np.testing.assert_array_equal(s.reshape(-1), golden_c1[f"{name}_s"])
