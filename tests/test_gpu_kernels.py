"""Parity of the sm_100a kernels (through the C-ABI) with the numpy oracle
and the reference's golden vectors.

Integer work (codes, scales, int32 accumulators) and every bf16/f16/f32
output is compared bit for bit: the kernels evaluate the same float32
expression sequence as the oracle.
"""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from conftest import cuda_ok
from oracle import qlinear_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module")
def P(pkg):
    return pkg


def dev(a, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dt is not None:
        t = t.to(TDT[dt])
    return t.cuda()


def host_f32(t):
    return t.float().cpu().numpy()


def bits(dt, v):
    v = np.asarray(v, np.float32)
    if dt == "bf16":
        return O.f32_to_bf16_bits(v)
    if dt == "f16":
        return v.astype(np.float16).view(np.uint16)
    return v.view(np.uint32)


def tbits(t):
    if t.dtype == torch.float32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


# ---------------------------------------------------------------------------
# (a) activation quantisation
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_quant_int8_golden(P, golden, dt):
    x = gi.activation(0, 37, 256, dt, zero_row=5)
    q, s = P.ops.quant_act_int8(dev(x, dt))
    np.testing.assert_array_equal(q.cpu().numpy(), golden[f"q8_{dt}_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), golden[f"q8_{dt}_s"])


def test_quant_int8_configs0_scale(P, golden):
    x = gi.activation(0, 4096, 3072, "bf16")
    q, s = P.ops.quant_act_int8(dev(x, "bf16"))
    import hashlib
    assert hashlib.sha256(q.cpu().numpy().tobytes()).hexdigest() == str(golden["q8_c0_q_sha"])
    np.testing.assert_array_equal(s.cpu().numpy(), golden["q8_c0_s"])


@pytest.mark.parametrize("K", [100, 250, 7])
def test_quant_int8_unaligned_rows(P, K):
    x = gi.activation(11, 19, K, "bf16")
    q, s = P.ops.quant_act_int8(dev(x, "bf16"))
    qo, so = O.quantize_int8_axiswise(x, -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_quant_int8_strided_rows(P):
    x = gi.activation(12, 40, 512, "bf16")
    xt = dev(x, "bf16")[:, :384]  # row stride 512, 16-byte aligned rows
    q, s = P.ops.quant_act_int8(xt)
    qo, so = O.quantize_int8_axiswise(x[:, :384], -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_quant_int8_long_rows(P):
    x = gi.activation(13, 8, 24576, "bf16")  # two chunks per thread
    q, s = P.ops.quant_act_int8(dev(x, "bf16"))
    qo, so = O.quantize_int8_axiswise(x, -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


ROTS = [("regular", 16), ("regular", 64), ("regular", 256), ("sylvester", 32), ("sylvester", 128)]


@pytest.mark.parametrize("kind,g", ROTS)
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_rotate_matches_oracle(P, kind, g, dt):
    x = gi.activation(14, 33, 1024, dt)
    y = P.ops.rotate(dev(x, dt), kind, g)
    yo = O.rotate(x, g, kind, dt)
    np.testing.assert_array_equal(tbits(y), bits(dt, yo))


@pytest.mark.parametrize("kind,g", ROTS)
def test_fused_rotate_quant_int8(P, kind, g):
    x = gi.activation(15, 64, 3072, "bf16")
    q, s = P.ops.quant_act_int8(dev(x, "bf16"), (kind, g))
    qo, so = O.quantize_int8_axiswise(O.rotate(x, g, kind, "bf16"), -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_fused_rotate_quant_long_rows(P):
    x = gi.activation(16, 4, 24576, "bf16")
    q, s = P.ops.quant_act_int8(dev(x, "bf16"), ("regular", 256))
    qo, so = O.quantize_int8_axiswise(O.rotate(x, 256, "regular", "bf16"), -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


# Row lengths 1024..16384 exercise the activation kernel's one-, two- and four-chunk forms: 64 chunks
# (smallest), 65 (odd: the last thread has one chunk), 193, 1024 (largest).
PAIR_CASES = [(1024, None), (1040, None), (3088, ("regular", 16)), (16384, None), (1024, ("sylvester", 32)),
              (1024, ("regular", 64)), (16384, ("regular", 256)), (16384, ("sylvester", 128)), (1040, ("regular", 16))]


@pytest.mark.parametrize("K,rot", PAIR_CASES)
@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_quant_int8_paired_chunks(P, K, rot, dt):
    x = gi.activation(17, 45, K, dt, zero_row=3)
    q, s = P.ops.quant_act_int8(dev(x, dt), rot)
    xr = x if rot is None else O.rotate(x, rot[1], rot[0], dt)
    qo, so = O.quantize_int8_axiswise(xr, -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


@pytest.mark.parametrize("K", [256, 2048, 24576])  # one-chunk, two-chunk-pair and long-row kernels
def test_quant_int8_round_half_even_ties(P, K):
    # scale 1.0 (absmax 127): codes of exact halves must round to even
    rng = np.random.default_rng(19)
    halves = np.float32(0.5) + rng.integers(-127, 127, size=(6, K)).astype(np.float32)
    x = np.clip(halves, -126.5, 126.5)
    x[:, 0] = 127.0
    q, s = P.ops.quant_act_int8(dev(x, "bf16"))
    qo, so = O.quantize_int8_axiswise(O.rnd("bf16", x), -1)
    assert np.all(so == 1.0)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)


@pytest.mark.parametrize("rot", [None, ("sylvester", 128)])
def test_quant_int8_paired_nonfinite_rows(P, rot):
    x = gi.activation(18, 9, 2048, "bf16")
    x[1, 100] = np.inf
    x[4, 2047] = -np.inf
    x[6, 1500] = np.nan
    q, s = P.ops.quant_act_int8(dev(x, "bf16"), rot)
    qo, so = O.quantize_int8_axiswise(x if rot is None else O.rotate(x, 128, "sylvester", "bf16"), -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)  # NaN matches NaN, Inf matches Inf


# Sylvester 128 with 64-element strips (a group over a lane pair; K <= 8192):
# K = 128 (two threads per row, 64 rows per CTA), 384 and 640 (CTAs whose
# last warp is partial), 1152, 3072 (the headline row) and 8192 (the largest
# that takes this form); zero, Inf and NaN rows; row count not a multiple of
# the rows per CTA.
@pytest.mark.parametrize("K", [128, 384, 640, 1152, 3072, 8192])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_quant_sylvester128_half_strips(P, K, dt):
    x = gi.activation(20 + K // 128, 75, K, dt)
    x[3] = 0.0
    x[10, K // 3] = np.inf
    x[17, K - 1] = -np.inf
    x[40, 5] = np.nan
    q, s = P.ops.quant_act_int8(dev(x, dt), ("sylvester", 128))
    qo, so = O.quantize_int8_axiswise(O.rotate(x, 128, "sylvester", dt), -1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_rotate_vs_reference_golden(P, golden):
    # the reference's own bf16 matmul rotation: within 1 bf16 ulp
    x = gi.activation(4, 32, 1024, "bf16")
    for name, g, kind in [("rot_reg256", 256, "regular"), ("rot_syl128", 128, "sylvester")]:
        y = tbits(P.ops.rotate(dev(x, "bf16"), kind, g)).astype(np.int32)
        d = np.abs(y - golden[f"{name}_y"].astype(np.int32))
        assert d.max() <= 1


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_quant_int4_rowwise(P, golden, dt):
    x = gi.activation(6, 37, 512, dt, zero_row=3)
    q, s = P.ops.quant_act_int4(dev(x, dt))
    qo, so = O.quantize_signed_int4_rowwise(x, dt)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    if dt == "f16":
        np.testing.assert_array_equal(q.cpu().numpy()[np.arange(37) != 3], golden["i4_f16_q"][np.arange(37) != 3])


def test_quant_int4_rowwise_reference_rotated_input(P, golden):
    xr = O.bf16_bits_to_f32(golden["i4_xrot"]).reshape(37, 512)
    q, s = P.ops.quant_act_int4(dev(xr, "bf16"))
    np.testing.assert_array_equal(q.cpu().numpy(), golden["i4_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), golden["i4_s"])


@pytest.mark.parametrize("kind,g", [("regular", 256), ("sylvester", 128)])
def test_fused_rotate_quant_int4(P, kind, g):
    x = gi.activation(17, 48, 3072, "bf16")
    q, s = P.ops.quant_act_int4(dev(x, "bf16"), (kind, g))
    qo, so = O.quantize_signed_int4_rowwise(O.rotate(x, g, kind, "bf16"), "bf16")
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_quant_int4_group128(P):
    x = gi.activation(18, 40, 3072, "bf16")
    q, s = P.ops.quant_act_int4(dev(x, "bf16"), ("sylvester", 128), group=128)
    qo, so = O.quantize_signed_int4_grouped(O.rotate(x, 128, "sylvester", "bf16"), "bf16")
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


# ---------------------------------------------------------------------------
# (b) W8A8 GEMM
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("M,N,K", [(37, 512, 256), (256, 384, 3072), (200, 300, 160), (129, 136, 96),
                                   (1, 8, 16), (513, 1024, 1024)])
def test_int_mm(P, M, N, K):
    rng = np.random.default_rng(M * 7 + N)
    a = rng.integers(-128, 128, (M, K), dtype=np.int8)
    w = rng.integers(-128, 128, (N, K), dtype=np.int8)
    c = P.ops.int_mm(dev(a), dev(w))
    np.testing.assert_array_equal(c.cpu().numpy(), O.int_mm(a, w))


def test_int_mm_k_padding(P):
    rng = np.random.default_rng(5)
    a = rng.integers(-128, 128, (33, 100), dtype=np.int8)
    w = rng.integers(-128, 128, (70, 100), dtype=np.int8)
    np.testing.assert_array_equal(P.ops.int_mm(dev(a), dev(w)).cpu().numpy(), O.int_mm(a, w))


def test_int_mm_extremes(P):
    # all -128 * -128 over K = 8192: 134217728 fits int32 exactly
    a = np.full((128, 8192), -128, np.int8)
    w = np.full((256, 8192), -128, np.int8)
    c = P.ops.int_mm(dev(a), dev(w)).cpu().numpy()
    assert (c == 128 * 128 * 8192).all()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_w8a8_golden(P, golden, dt):
    x = gi.activation(1, 37, 256, dt)
    wq, ws = golden[f"w8_{dt}_wq"], golden[f"w8_{dt}_ws"]
    b = gi.bias(1, 512, dt)
    xq, xs = P.ops.quant_act_int8(dev(x, dt))
    y = P.ops.gemm_w8a8(xq, xs, dev(wq), dev(ws), dev(b, dt), TDT[dt], per_row=True)
    np.testing.assert_array_equal(tbits(y), golden[f"w8_{dt}_y"])
    y0 = P.ops.gemm_w8a8(xq, xs, dev(wq), dev(ws), None, TDT[dt], per_row=True)
    np.testing.assert_array_equal(tbits(y0), golden[f"w8_{dt}_y_nobias"])


def test_w8a8_medium_golden(P, golden):
    x = gi.activation(2, 256, 3072, "bf16")
    w = gi.weight(2, 384, 3072)
    wq, ws = P.ops.quant_weight_int8(dev(w))
    np.testing.assert_array_equal(ws.cpu().numpy(), golden["w8m_ws"])
    xq, xs = P.ops.quant_act_int8(dev(x, "bf16"))
    y = P.ops.gemm_w8a8(xq, xs, wq, ws, dev(gi.bias(2, 384, "bf16"), "bf16"), torch.bfloat16)
    np.testing.assert_array_equal(tbits(y), golden["w8m_y"])


def test_w8a8_tensorwise_golden(P, golden):
    x = gi.activation(3, 37, 256, "f16")
    wq = gi.int8_weight(3, 512, 256)
    xq, xs = P.ops.quant_act_int8(dev(x, "f16"))
    y = P.ops.gemm_w8a8(xq, xs, dev(wq), torch.tensor([0.01]), dev(gi.bias(3, 512, "f16"), "f16"),
                        torch.float16, per_row=False)
    np.testing.assert_array_equal(tbits(y), golden["w8t_y"])


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("M,N,K", [(300, 520, 512), (1024, 3072, 3072)])
def test_w8a8_vs_oracle(P, dt, M, N, K):
    x = gi.activation(20, M, K, dt)
    w = gi.weight(20, N, K)
    b = gi.bias(20, N, dt)
    wq, ws = O.quantize_int8_axiswise(w, 1)
    xq, xs = P.ops.quant_act_int8(dev(x, dt))
    y = P.ops.gemm_w8a8(xq, xs, dev(wq), dev(ws), dev(b, dt), TDT[dt])
    yo = O.int8_forward_dynamic_per_row(x, wq, ws, b, dt)
    np.testing.assert_array_equal(tbits(y), bits(dt, yo))


@pytest.mark.parametrize("g,kind", [(256, "regular"), (128, "sylvester")])
def test_convrot_w8a8_linear_configs1_shape(P, g, kind):
    """ConvRot W8A8 at M=1024, N=3072, K=3072 (outlier activations)."""
    M, N, K = 1024, 3072, 3072
    x = gi.activation(1, M, K, "bf16")
    w = gi.weight(1, N, K)
    b = gi.bias(1, N, "bf16")
    wq, ws = O.quantize_weight_int8(w, g, kind)
    gq, gs = P.ops.quant_weight_int8(dev(w), (kind, g))
    np.testing.assert_array_equal(gq.cpu().numpy(), wq)
    np.testing.assert_array_equal(gs.cpu().numpy(), ws)
    xq, xs = P.ops.quant_act_int8(dev(x, "bf16"), (kind, g))
    y = P.ops.gemm_w8a8(xq, xs, gq, gs, dev(b, "bf16"), torch.bfloat16)
    xo = O.rotate(x, g, kind, "bf16")
    yo = O.int8_forward_dynamic_per_row(xo, wq, ws, b, "bf16")
    np.testing.assert_array_equal(tbits(y), bits("bf16", yo))


# ---------------------------------------------------------------------------
# (c) packed-INT4 GEMMs
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("M,N,K", [(37, 128, 512), (256, 384, 3072), (130, 264, 160)])
def test_int4_mm(P, M, N, K):
    rng = np.random.default_rng(N)
    a = rng.integers(-7, 8, (M, K), dtype=np.int8)
    wn = rng.integers(-8, 8, (N, K), dtype=np.int8)
    wp = O.pack_int4_row_major(wn)
    c = P.ops.int4_mm(dev(a), dev(wp))
    np.testing.assert_array_equal(c.cpu().numpy(), O.int_mm(a, wn))


def test_w4a4_forward_golden(P, golden):
    x = gi.activation(9, 37, 512, "bf16")
    b = gi.bias(9, 128, "bf16")
    pw, ps = golden["i4w_packed"], golden["i4w_scale"]
    qa, sa = P.ops.quant_act_int4(dev(x, "bf16"), ("regular", 256))
    acc = P.ops.int4_mm(qa, dev(pw))
    np.testing.assert_array_equal(acc.cpu().numpy(), golden["i4fwd_acc"])
    y = P.ops.gemm_w4a4(qa, sa, dev(pw), dev(ps), dev(b, "bf16"), torch.bfloat16)
    np.testing.assert_array_equal(tbits(y), golden["i4fwd_y"])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_w4a4_vs_oracle(P, dt):
    M, N, K = 300, 640, 3072
    x = gi.activation(21, M, K, dt)
    w = gi.weight(21, N, K)
    b = gi.bias(21, N, dt)
    pw, ps = O.quantize_convrot_w4a4_weight(w, 256, "regular")
    gp, gs = P.ops.quant_weight_int4(dev(w), ("regular", 256))
    np.testing.assert_array_equal(gp.cpu().numpy(), pw)
    np.testing.assert_array_equal(gs.cpu().numpy(), ps)
    qa, sa = P.ops.quant_act_int4(dev(x, dt), ("regular", 256))
    y = P.ops.gemm_w4a4(qa, sa, gp, gs, dev(b, dt), TDT[dt])
    yo = O.convrot_w4a4_forward(x, pw, ps, b, 256, "regular", dt)
    np.testing.assert_array_equal(tbits(y), bits(dt, yo))


def _w4a4_case(seed, M, N, K, with_bias, dt):
    rng = np.random.default_rng(seed)
    qa = rng.integers(-8, 8, (M, K), dtype=np.int8)
    wn = rng.integers(-8, 8, (N, K), dtype=np.int8)
    sa = (rng.random(M) * 0.02 + 1e-3).astype(np.float32)
    ws = (rng.random(N) * 0.02 + 1e-3).astype(np.float32)
    b = O.rnd(dt, rng.standard_normal(N).astype(np.float32)) if with_bias else None
    return qa, wn, sa, ws, b


# Row-wise W4A4 GEMM on ragged M, N and K tails (partial tiles in every
# dimension, a K tail inside one 128-deep step), every output dtype, rows
# that are not 16-byte aligned (N = 1028 in bf16), with and without bias
@pytest.mark.parametrize("M,N,K,with_bias,dt", [(513, 264, 160, True, "bf16"), (256, 256, 128, False, "f16"),
                                                 (600, 1000, 1024, True, "f32"), (1024, 3072, 3072, True, "bf16"),
                                                 (300, 1028, 384, True, "bf16"), (255, 640, 512, True, "bf16"),
                                                 (700, 200, 256, False, "f16")])
def test_w4a4_rowwise_shapes(P, M, N, K, with_bias, dt):
    qa, wn, sa, ws, b = _w4a4_case(M + N + K, M, N, K, with_bias, dt)
    pw = O.pack_int4_row_major(wn)
    y = P.ops.gemm_w4a4(dev(qa), torch.from_numpy(sa).cuda(), dev(pw), torch.from_numpy(ws).cuda(),
                        None if b is None else dev(b, dt), TDT[dt])
    yo = O.w4a4_rowwise_epilogue(O.int_mm(qa, wn), sa, ws, b, dt)
    np.testing.assert_array_equal(tbits(y), bits(dt, yo))
    assert P.ops.device_error() == 0


def test_w4a4_rowwise_full_size_rows(P):
    # Packed-INT4 W4A4 linear, M=4096 N=12288 K=3072, seed 5: whole GEMM on
    # the GPU, oracle on a sample of rows (rows are independent)
    M, N, K = 4096, 12288, 3072
    qa, wn, sa, ws, b = _w4a4_case(5, M, N, K, True, "bf16")
    pw = O.pack_int4_row_major(wn)
    y = P.ops.gemm_w4a4(dev(qa), torch.from_numpy(sa).cuda(), dev(pw), torch.from_numpy(ws).cuda(), dev(b, "bf16"),
                        torch.bfloat16)
    rows = _rows_sample(M, seed=2)
    yo = O.w4a4_rowwise_epilogue(O.int_mm(qa[rows], wn), sa[rows], ws, b, "bf16")
    np.testing.assert_array_equal(tbits(y)[rows], bits("bf16", yo))


# ---------------------------------------------------------------------------
# (c) group-128 int4-weight GEMMs (W4A8, W4A4)
# ---------------------------------------------------------------------------

G128_SHAPES = [(37, 128, 128), (300, 520, 512), (130, 300, 384), (256, 384, 3072)]


def _g128_weight(P, seed, N, K, rot=None):
    """bf16 weight, optional rotation, symmetric int4 per-group-128 in bf16
    math; kernel output checked against the oracle quantiser."""
    w = O.rnd("bf16", gi.weight(seed, N, K))
    wr = w if rot is None else O.rotate(w, rot[1], rot[0], "bf16")
    qo, so = O.quantize_signed_int4_grouped(wr, "bf16")
    gp, gs = P.ops.quant_weight_int4(dev(w, "bf16"), rot, group=128)
    np.testing.assert_array_equal(gp.cpu().numpy(), O.pack_int4_row_major(qo))
    np.testing.assert_array_equal(gs.cpu().numpy(), so)
    return gp, gs


@pytest.mark.parametrize("M,N,K", G128_SHAPES)
@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_w4a8_g128_vs_oracle(P, M, N, K, dt):
    x = gi.activation(30, M, K, dt)
    b = gi.bias(30, N, dt) if dt != "f16" else None
    gp, gs = _g128_weight(P, 30, N, K)
    qa, sa = P.ops.quant_act_int8(dev(x, dt))
    y = P.ops.gemm_w4_g128(qa, sa, gp, gs, None if b is None else dev(b, dt), TDT[dt])
    yo = O.w4a8_g128_forward_from_q(qa.cpu().numpy(), sa.cpu().numpy(), gp.cpu().numpy(), gs.cpu().numpy(), b, dt)
    np.testing.assert_array_equal(tbits(y), bits(dt, yo))


@pytest.mark.parametrize("M,N,K", G128_SHAPES)
@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_w4a4_g128_vs_oracle(P, M, N, K, dt):
    rot = ("sylvester", 128)
    x = gi.activation(31, M, K, dt)
    b = gi.bias(31, N, dt)
    gp, gs = _g128_weight(P, 31, N, K, rot)
    qa, sa = P.ops.quant_act_int4(dev(x, dt), rot, group=128)
    y = P.ops.gemm_w4_g128(qa, sa, gp, gs, dev(b, dt), TDT[dt], a_int4_groups=True)
    yo = O.w4a4_g128_forward_from_q(qa.cpu().numpy(), sa.cpu().numpy(), gp.cpu().numpy(), gs.cpu().numpy(), b, dt)
    np.testing.assert_array_equal(tbits(y), bits(dt, yo))


def _rows_sample(M, n=48, seed=0):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, M - 1], rng.choice(M, n, replace=False)]))


def test_w4a8_g128_full_size_rows(P):
    # Packed-INT4 W4A8 linear, M=4096 N=12288 K=3072, seed 2: whole GEMM on
    # the GPU, oracle on a sample of rows (rows are independent)
    M, N, K = 4096, 12288, 3072
    x = gi.activation(2, M, K, "bf16")
    gp, gs = P.ops.quant_weight_int4(dev(O.rnd("bf16", gi.weight(2, N, K)), "bf16"), None, group=128)
    qa, sa = P.ops.quant_act_int8(dev(x, "bf16"))
    b = gi.bias(2, N, "bf16")
    y = P.ops.gemm_w4_g128(qa, sa, gp, gs, dev(b, "bf16"), torch.bfloat16)
    rows = _rows_sample(M)
    yo = O.w4a8_g128_forward_from_q(qa.cpu().numpy()[rows], sa.cpu().numpy()[rows], gp.cpu().numpy(),
                                    gs.cpu().numpy(), b, "bf16")
    np.testing.assert_array_equal(tbits(y)[rows], bits("bf16", yo))


@pytest.mark.parametrize("N", [3072, 12288])
def test_w4a4_g128_full_size_rows(P, N):
    # Packed-INT4 W4A4 linear with ConvRot (Sylvester 128), M=4096, K=3072, seed 3
    M, K = 4096, 3072
    rot = ("sylvester", 128)
    x = gi.activation(3, M, K, "bf16")
    gp, gs = P.ops.quant_weight_int4(dev(O.rnd("bf16", gi.weight(3, N, K)), "bf16"), rot, group=128)
    qa, sa = P.ops.quant_act_int4(dev(x, "bf16"), rot, group=128)
    b = gi.bias(3, N, "bf16")
    y = P.ops.gemm_w4_g128(qa, sa, gp, gs, dev(b, "bf16"), torch.bfloat16, a_int4_groups=True)
    rows = _rows_sample(M, seed=1)
    yo = O.w4a4_g128_forward_from_q(qa.cpu().numpy()[rows], sa.cpu().numpy()[rows], gp.cpu().numpy(),
                                    gs.cpu().numpy(), b, "bf16")
    np.testing.assert_array_equal(tbits(y)[rows], bits("bf16", yo))


def test_g128_rejects_bad_k(P):
    a = torch.zeros((16, 192), dtype=torch.int8, device="cuda")
    w = torch.zeros((16, 96), dtype=torch.int8, device="cuda")
    with pytest.raises(Exception):
        P.ops.gemm_w4_g128(a, torch.ones(16, device="cuda"), w, torch.ones((16, 1), device="cuda"))


# ---------------------------------------------------------------------------
# (d) weight-side kernels
# ---------------------------------------------------------------------------


def test_requant_asym_w4a8_golden(P, golden):
    packed, cb, sch, srel = gi.asym_w4a8(10, 96, 256, 16)
    q, s = P.ops.requant_asym_w4a8(dev(packed), dev(cb), dev(sch), dev(srel), 16)
    np.testing.assert_array_equal(q.cpu().numpy(), golden["w4a8_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), golden["w4a8_s"])


def test_dequant_asym_w4a8_golden(P, golden):
    # the reference's own float dequantisation (w4a8_int8.py:46-75), bit for bit
    packed, cb, sch, srel = gi.asym_w4a8(10, 96, 256, 16)
    w = P.w4a8_int8.dequant_asym_w4a8_to_float(dev(packed), dev(cb), dev(sch), dev(srel), 16)
    np.testing.assert_array_equal(w.cpu().numpy().view(np.uint32), golden["w4a8_deq"].view(np.uint32))
    with pytest.raises(ValueError):
        P.ops.dequant_asym_w4a8(dev(packed), dev(cb), dev(sch), dev(srel), 32)


@pytest.mark.parametrize("wdt", ["bf16", "f16", "f32"])
def test_quant_weight_int8_dtypes(P, wdt):
    w = O.rnd(wdt, gi.weight(22, 96, 1024))
    q, s = P.ops.quant_weight_int8(dev(w, wdt), ("regular", 256))
    qo, so = O.quantize_weight_int8(w, 256, "regular")
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_lora_dequant_requant(P, golden):
    oq, os_ = golden["otf_q"], golden["otf_s"]
    wf = P.ops.dequant_int8(dev(oq), dev(os_), ("regular", 256))
    wo = O.dequant_unrotate_int8(oq, os_, 256, "regular")
    np.testing.assert_array_equal(host_f32(wf), wo)
    delta = gi.weight(12, 48, 512) * np.float32(0.05)
    patched = wo + delta
    q = P.ops.requant_int8(dev(patched), dev(os_), ("regular", 256))
    np.testing.assert_array_equal(q.cpu().numpy(), O.rotate_requant_int8(patched, os_, 256, "regular"))
    # no rotation, tensor-wide scale
    q2 = P.ops.requant_int8(dev(patched), 0.003)
    np.testing.assert_array_equal(q2.cpu().numpy(), O.quantize_int8(patched, np.float32(0.003)))


def test_stochastic_requant_distribution(P):
    x = np.full((64, 4096), 0.3, np.float32)
    q = P.ops.requant_int8(dev(x), 1.0, stochastic=True, seed=7).cpu().numpy()
    assert set(np.unique(q)) <= {0, 1}
    assert abs(q.mean() - 0.3) < 0.01
    q2 = P.ops.requant_int8(dev(x), 1.0, stochastic=True, seed=7).cpu().numpy()
    np.testing.assert_array_equal(q, q2)


# ---------------------------------------------------------------------------
# errors
# ---------------------------------------------------------------------------


def test_cpu_tensor_rejected(P):
    with pytest.raises(RuntimeError):
        P.ops.quant_act_int8(torch.zeros(4, 16, dtype=torch.bfloat16))


def test_bad_group_rejected(P):
    from comfyui_int8_fast_rocm_b200._native import NativeError
    with pytest.raises(NativeError):
        P.ops.quant_act_int8(torch.zeros(4, 96, dtype=torch.bfloat16, device="cuda"), ("regular", 64))


def test_empty_inputs(P):
    q, s = P.ops.quant_act_int8(torch.zeros(0, 256, dtype=torch.bfloat16, device="cuda"))
    assert q.shape == (0, 256) and s.shape == (0, 1)
    y = P.ops.gemm_w8a8(q, s, torch.zeros(64, 256, dtype=torch.int8, device="cuda"),
                        torch.ones(64, 1, device="cuda"), None, torch.bfloat16)
    assert y.shape == (0, 64)


def test_no_device_error_flag(P):
    torch.cuda.synchronize()
    assert P.ops.device_error() == 0


# ---------------------------------------------------------------------------
# SiTU input activation (floating point: tolerance vs a float64 evaluation)
# ---------------------------------------------------------------------------


def _situ_ref(x64):
    K = x64.shape[-1] // 2
    h, g = x64[..., :K], x64[..., K:]
    return 4 * np.tanh(g / 4) / (1 + np.exp(-g)) * 25 * np.tanh(h / 25)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_situ(P, dt):
    rng = np.random.default_rng(3)
    x = O.rnd(dt, rng.standard_normal((37, 2 * 200), dtype=np.float32) * np.float32(6.0))
    x[0, :8] = np.float32(1e-3)  # the small-|x| polynomial branch
    y = host_f32(P.ops.situ(dev(x, dt)))
    ref = _situ_ref(x.astype(np.float64))
    if dt == "f32":
        np.testing.assert_allclose(y, ref, rtol=2e-6, atol=1e-7)
    else:  # one rounding to bf16 of a float32 result: within 1 bf16 ulp
        ulp = np.spacing(np.abs(ref).astype(np.float32)) * 2 ** 16
        assert (np.abs(y - ref) <= ulp + 1e-30).all()


# ---------------------------------------------------------------------------
# the W8A8 linear at the benchmarked shapes (whole problem on the GPU, the
# oracle on a sample of rows: rows of a linear are independent)
# ---------------------------------------------------------------------------

BENCH_SHAPES = [
    # (M, N, K, rotation, seed)
    (4096, 12288, 3072, ("sylvester", 128), 1),  # the ConvRot W8A8 headline
    (8192, 9216, 12288, ("sylvester", 128), 1),
    (4096, 3072, 12288, ("regular", 256), 1),
    (4096, 3072, 3072, None, 0),  # the plain dynamic W8A8 linear, no rotation
]


@pytest.mark.parametrize("M,N,K,rot,seed", BENCH_SHAPES)
def test_w8a8_linear_bench_shapes_rows(P, M, N, K, rot, seed):
    """Codes, scales and bf16 outputs of the plain CTA-pair W8A8 kernel (6
    operand stages, double TMEM accumulator, several tiles per cluster) at
    the benchmarked shapes, against the oracle on 50 rows."""
    x = gi.activation(seed, M, K, "bf16")
    w = gi.weight(seed, N, K)
    b = gi.bias(seed, N, "bf16")
    gq, gs = P.ops.quant_weight_int8(dev(w), rot)
    wrows = _rows_sample(N, n=16, seed=seed + 7)
    wq_o, ws_o = O.quantize_weight_int8(w[wrows], *((rot[1], rot[0]) if rot else ()))
    np.testing.assert_array_equal(gq.cpu().numpy()[wrows], wq_o)
    np.testing.assert_array_equal(gs.cpu().numpy()[wrows], ws_o)
    xq, xs = P.ops.quant_act_int8(dev(x, "bf16"), rot)
    y = P.ops.gemm_w8a8(xq, xs, gq, gs, dev(b, "bf16"), torch.bfloat16)
    assert P.ops.device_error() == 0
    rows = _rows_sample(M, seed=seed + 11)
    xr = x[rows] if rot is None else O.rotate(x[rows], rot[1], rot[0], "bf16")
    qo, so = O.quantize_int8_axiswise(xr, -1)
    np.testing.assert_array_equal(xq.cpu().numpy()[rows], qo)
    np.testing.assert_array_equal(xs.cpu().numpy()[rows], so)
    yo = O.w8a8_epilogue_per_row(O.int_mm(qo, gq.cpu().numpy()), so, gs.cpu().numpy(), b, "bf16")
    np.testing.assert_array_equal(tbits(y)[rows], bits("bf16", yo))


# A last wave of at most half the CTA pairs runs as 128-column units: 768
# tiles = 10 waves of 74 + 28 (4096 x 12288, the headline grid; and 4000 x
# 12160, whose last row block and last column tile are partial, so one
# narrow unit lies wholly past N), full output rows against the oracle,
# including the last row.
@pytest.mark.parametrize("M,N,K", [(4096, 12288, 1024), (4000, 12160, 1024)])
def test_w8a8_narrow_last_wave_rows(P, M, N, K):
    rng = np.random.default_rng(M + N)
    a = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    sa = (rng.random(M, dtype=np.float32) * 0.02 + 1e-3).astype(np.float32)
    sw = (rng.random(N, dtype=np.float32) * 0.002 + 1e-4).astype(np.float32)
    b = O.rnd("bf16", rng.standard_normal(N).astype(np.float32) * 0.5)
    y = P.ops.gemm_w8a8(dev(a), torch.from_numpy(sa).cuda(), dev(w), torch.from_numpy(sw).cuda(), dev(b, "bf16"),
                        torch.bfloat16)
    assert P.ops.device_error() == 0
    rows = np.unique(np.concatenate([_rows_sample(M, seed=5), [M - 1, M // 2, 2048, 3071]]))
    yo = O.w8a8_epilogue_per_row(O.int_mm(a[rows], w), sa[rows], sw, b, "bf16")
    np.testing.assert_array_equal(tbits(y)[rows], bits("bf16", yo))


@pytest.mark.parametrize("name,K,g,kind", [("syl128_k3072", 3072, 128, "sylvester"),
                                           ("reg256_k3072", 3072, 256, "regular"),
                                           ("syl128_k12288", 12288, 128, "sylvester")])
def test_rotated_codes_vs_reference_full_size(P, golden_c1, name, K, g, kind):
    """Activation codes of the fused rotate+quantise kernel against the
    reference's own rotate_activation + quantize_int8_axiswise on the
    4096-token activations of the ConvRot linear.  The golden file lists
    where the reference's codes differ from the fixed-order butterfly's; the
    kernel's codes patched there must hash to the reference's digest, so the
    kernel differs from the reference at exactly those positions."""
    x = gi.activation(1, 4096, K, "bf16")
    q, s = P.ops.quant_act_int8(dev(x, "bf16"), (kind, g))
    qf = q.cpu().numpy().reshape(-1).copy()
    pos = golden_c1[f"{name}_diff_pos"]
    assert pos.size <= 2e-6 * qf.size  # 13 (K=3072) and 29 (K=12288) positions
    qf[pos] = golden_c1[f"{name}_diff_val"]
    import hashlib
    assert hashlib.sha256(qf.tobytes()).hexdigest() == str(golden_c1[f"{name}_q_sha"])
    differ = int((s.cpu().numpy().reshape(-1) != golden_c1[f"{name}_s"]).sum())
    assert differ == int(golden_c1[f"{name}_scale_rows_differ"]) == 0


# ---------------------------------------------------------------------------
# split K (small W8A8 problems): bit-equal to the unsplit kernel
# ---------------------------------------------------------------------------


def _unsplit_w8a8(P, xq, xs, wq, ws, b, out_dtype, per_row=True):
    """qlin_gemm_w8a8 called directly: the CTA-pair kernel without split K."""
    from comfyui_int8_fast_rocm_b200 import _native
    M, K = xq.shape
    Nn = wq.shape[0]
    out = torch.empty((M, Nn), dtype=out_dtype, device=xq.device)
    _native.call("qlin_gemm_w8a8", xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(),
           _native.WSCALE_ROW if per_row else _native.WSCALE_TENSOR, 0 if b is None else b.data_ptr(),
           out.data_ptr(),
           P.ops.dtype_code(out_dtype), M, Nn, K, torch.cuda.current_stream().cuda_stream)
    return out


def _scratch_bytes(M, N, K):
    import ctypes
    from comfyui_int8_fast_rocm_b200 import _native
    out = ctypes.c_uint64(0)
    _native.call("qlin_gemm_w8a8_splitk_scratch", M, N, K, ctypes.addressof(out))
    return int(out.value)


@pytest.mark.parametrize("M,N,K", [(512, 768, 8192), (300, 520, 8192), (256, 1024, 16384), (1024, 2048, 16384)])
@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_w8a8_splitk_equals_unsplit(P, M, N, K, dt):
    x = gi.activation(40, M, K, dt)
    w = gi.weight(40, N, K)
    b = dev(gi.bias(40, N, dt), dt)
    wq, ws = P.ops.quant_weight_int8(dev(w))
    xq, xs = P.ops.quant_act_int8(dev(x, dt))
    xs = xs.reshape(-1).contiguous()
    ws = ws.reshape(-1).contiguous()
    assert _scratch_bytes(M, N, K) > 0  # these shapes split
    want = _unsplit_w8a8(P, xq, xs, wq, ws, b, TDT[dt])
    for _ in range(2):  # the scratch's counters are reset by every call
        got = P.ops.gemm_w8a8(xq, xs, wq, ws, b, TDT[dt])
        np.testing.assert_array_equal(tbits(got), tbits(want))
    assert P.ops.device_error() == 0


def test_w8a8_splitk_tensorwise_and_no_bias(P):
    M, N, K = 512, 1024, 12288
    x = gi.activation(41, M, K, "bf16")
    wq = dev(np.random.default_rng(41).integers(-127, 128, (N, K), dtype=np.int8))
    ws = torch.tensor([0.0123], device="cuda")
    xq, xs = P.ops.quant_act_int8(dev(x, "bf16"))
    xs = xs.reshape(-1).contiguous()
    want = _unsplit_w8a8(P, xq, xs, wq, ws, None, torch.bfloat16, per_row=False)
    got = P.ops.gemm_w8a8(xq, xs, wq, ws, None, torch.bfloat16, per_row=False)
    np.testing.assert_array_equal(tbits(got), tbits(want))


def test_w8a8_splitk_rows_vs_oracle(P):
    """A split problem with rotation (three K parts of 64 slabs) against the
    oracle on sampled rows."""
    M, N, K = 768, 1536, 24576
    x = gi.activation(42, M, K, "bf16")
    w = gi.weight(42, N, K)
    b = gi.bias(42, N, "bf16")
    gq, gs = P.ops.quant_weight_int8(dev(w), ("sylvester", 128))
    xq, xs = P.ops.quant_act_int8(dev(x, "bf16"), ("sylvester", 128))
    y = P.ops.gemm_w8a8(xq, xs, gq, gs, dev(b, "bf16"), torch.bfloat16)
    rows = _rows_sample(M, seed=43)
    yo = O.w8a8_epilogue_per_row(O.int_mm(xq.cpu().numpy()[rows], gq.cpu().numpy()), xs.cpu().numpy()[rows],
                                 gs.cpu().numpy(), b, "bf16")
    np.testing.assert_array_equal(tbits(y)[rows], bits("bf16", yo))


def test_w8a8_large_problem_does_not_split(P):
    assert _scratch_bytes(4096, 12288, 3072) == 0
    assert _scratch_bytes(8192, 9216, 12288) == 0
    assert _scratch_bytes(1024, 3072, 3072) == 0  # measured slower split (partial traffic)


# Regular-256 rotation + int8 on problems of 2^25 elements and more, which the
# launcher sends to the strip kernel (a group across a lane pair), against
# the oracle on sampled rows, with zero and non-finite rows.
@pytest.mark.parametrize("M,K,dt", [(16384, 3072, "bf16"), (2816, 12288, "f16")])
def test_quant_regular256_large_rows(P, M, K, dt):
    x = gi.activation(50 + K, M, K, dt, zero_row=7)
    x[11, 5] = np.inf
    x[13, 100] = np.nan
    q, s = P.ops.quant_act_int8(dev(x, dt), ("regular", 256))
    rows = sorted(set(_rows_sample(M, seed=K).tolist()) | {7, 11, 13, M - 1})
    qo, so = O.quantize_int8_axiswise(O.rotate(x[rows], 256, "regular", dt), -1)
    np.testing.assert_array_equal(q.cpu().numpy()[rows], qo)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1)[rows], np.asarray(so, np.float32).reshape(-1))
    assert P.ops.device_error() == 0


# ---------------------------------------------------------------------------
# programmatic dependent launch: consumers read their producers' fresh data
# ---------------------------------------------------------------------------


def test_pdl_chain_reads_fresh_inputs(P):
    """The quantiser and the CTA-pair GEMM are launched with programmatic
    dependent launch.  A chain [copy new rows in] -> quantise -> GEMM, run 24
    times without synchronising, with four input batches in turn, must give
    each batch's eager result bit for bit -- a consumer that read its
    operands before its producer finished would see the previous batch --
    both enqueued directly and replayed from a CUDA graph."""
    torch.manual_seed(11)
    M, N, K = 2048, 3072, 3072
    rot = ("sylvester", 128)
    xs = [(torch.randn((M, K), device="cuda") * (1 + i)).to(torch.bfloat16) for i in range(4)]
    wq, ws = P.ops.quant_weight_int8((torch.randn((N, K), device="cuda") * 0.02).to(torch.bfloat16), rot)
    b = (torch.randn(N, device="cuda") * 0.01).to(torch.bfloat16)

    def linear(x):
        q, s = P.ops.quant_act_int8(x, rot)
        return P.ops.gemm_w8a8(q, s, wq, ws, b, torch.bfloat16)

    want = [linear(x).clone() for x in xs]
    torch.cuda.synchronize()
    xbuf = torch.empty_like(xs[0])
    outs = []
    for i in range(24):
        xbuf.copy_(xs[i % 4])
        outs.append(linear(xbuf))
    torch.cuda.synchronize()
    for i, y in enumerate(outs):
        assert torch.equal(y, want[i % 4]), i

    # the same chain captured once and replayed with new rows each time
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            linear(xbuf)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = linear(xbuf)
    for i in range(12):
        xbuf.copy_(xs[i % 4])
        g.replay()
        assert torch.equal(yg, want[i % 4]), i
    del g
    assert P.ops.device_error() == 0
