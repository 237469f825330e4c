"""Parity of the DiT-block kernels around the quantised linear that are not
the quantiser's prologue or the GEMM's epilogue (through the C-ABI):

* ``qlin_quant_act_int8_cat``: per-token int8 of a concatenated row read
  from its two parts -- bit-exact against the same quantisation of the
  materialised ``torch.cat`` and against the oracle;
* ``qlin_qk_norm_rope``: in-place q/k RMSNorm + float32 rotary embedding --
  bit-exact against the oracle on rows whose RMS statistic sums exactly in
  float32; on random rows (the statistic is summed in another order) within
  two units of the dtype times the head vector's largest value, with
  >= 99.9 % of elements bit-equal.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import cuda_ok
from oracle import qlinear_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
UNIT = {"bf16": 2.0 ** -7, "f16": 2.0 ** -10}


def dev(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a)).to(TDT[dt]).cuda()


def bits(t):
    t = t.cpu()
    return t.view(torch.int16).numpy() if t.element_size() == 2 else t.view(torch.int32).numpy()


ROTS = [None, ("regular", 256), ("sylvester", 128), ("regular", 16)]


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("rot", ROTS)
@pytest.mark.parametrize("M,K1,K2,pad1,pad2", [(37, 3072, 12288, 0, 64), (5, 16, 240, 8, 0), (64, 128, 128, 16, 16),
                                               (130, 1024, 2048, 0, 0), (3, 1536, 512, 24, 40)])
def test_quant_cat_matches_cat(pkg, dt, rot, M, K1, K2, pad1, pad2):
    if rot is not None and (K1 + K2) % rot[1]:
        pytest.skip("row length not a multiple of the rotation block")
    rng = np.random.default_rng(M + K1 + K2)
    a = rng.standard_normal((M, K1 + pad1)).astype(np.float32) * 2
    b = rng.standard_normal((M, K2 + pad2)).astype(np.float32)
    b[:, rng.integers(0, K2, 3)] *= 20  # outlier channels
    ta, tb = dev(a, dt), dev(b, dt)
    x1, x2 = ta[:, pad1:], tb[:, :K2]  # strided views (row pitch K + pad)
    q, s = pkg.ops.quant_act_int8_cat(x1, x2, rot)
    q_ref, s_ref = pkg.ops.quant_act_int8(torch.cat((x1, x2), -1), rot)
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref)
    np.testing.assert_array_equal(bits(s), bits(s_ref))
    xo = np.concatenate([O.rnd(dt, a)[:, pad1:], O.rnd(dt, b)[:, :K2]], 1) if dt != "f32" else \
        np.concatenate([a[:, pad1:], b[:, :K2]], 1)
    if rot is not None:
        xo = O.rotate(xo, rot[1], rot[0], dt)
    qo, so = O.quantize_int8_axiswise(xo, dim=-1)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.astype(np.float32).view(np.uint32))
    assert pkg.ops.device_error() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_quant_cat_large_regular256(pkg, dt):
    """A single block's linear2 input at a size that takes the strip kernel
    (regular 256, >= 2^25 elements): 2200 rows of [attention 3072 | MLP
    12288] with a padded MLP row pitch; equal to quantising torch.cat of the
    parts, and to the oracle on 24 sampled rows plus the first and last."""
    M, K1, K2 = 2200, 3072, 12288
    g = torch.Generator(device="cuda").manual_seed(9)
    ta = torch.randn((M, K1), generator=g, device="cuda").to(TDT[dt])
    tb = (torch.randn((M, K2 + 64), generator=g, device="cuda") * 0.5).to(TDT[dt])
    tb[:, 77] *= 20
    ta[5] = 0.0
    x2 = tb[:, :K2]
    rot = ("regular", 256)
    q, s = pkg.ops.quant_act_int8_cat(ta, x2, rot)
    q_ref, s_ref = pkg.ops.quant_act_int8(torch.cat((ta, x2), -1), rot)
    assert torch.equal(q, q_ref)
    np.testing.assert_array_equal(bits(s), bits(s_ref))
    rows = np.unique(np.concatenate([[0, 5, M - 1], np.random.default_rng(3).integers(0, M, 24)]))
    xo = torch.cat((ta, x2), -1)[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    qo, so = O.quantize_int8_axiswise(O.rotate(xo, 256, "regular", dt), dim=-1)
    np.testing.assert_array_equal(q.cpu().numpy()[rows], qo)
    np.testing.assert_array_equal(s.cpu().numpy()[rows].view(np.uint32), so.astype(np.float32).view(np.uint32))
    assert pkg.ops.device_error() == 0


def test_quant_cat_rejects_misaligned(pkg):
    a = torch.zeros((4, 40), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((4, 32), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(pkg._native.NativeError):
        pkg._native.call("qlin_quant_act_int8_cat", a.data_ptr(), 40, 24, b.data_ptr(), 32, 32, 0, 4, 0, 0, 0.0,
                         b.data_ptr(), b.data_ptr(), torch.cuda.current_stream().cuda_stream)


def heads_close(got, ref, H, hd, dt):
    """Per q/k head vector: |got - ref| <= 2 units of the dtype times the
    vector's largest |value|.  A normalised value whose rounding flipped by
    one unit moves each rotated pair by at most one unit of that value (the
    rotation keeps a pair's length), and the output rounding adds one unit
    of the output."""
    g = np.asarray(got, np.float64)[:, :2 * H * hd].reshape(-1, 2 * H, hd)
    r = np.asarray(ref, np.float64)[:, :2 * H * hd].reshape(-1, 2 * H, hd)
    tol = 2 * UNIT[dt] * np.maximum(np.abs(r).max(-1, keepdims=True), 2.0 ** -20)
    return bool(np.all(np.abs(g - r) <= tol))


def rope_tables(L, hd):
    inv = 1.0 / (10000.0 ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    ang = np.arange(L, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def exact_heads(rng, R, C, dt):
    """Multiples of 1/8 in [-4, 4]: every float32 partial sum of squares of a
    128-element head vector is exact (<= 128 * 16, 1/64 steps), so the RMS
    statistic does not depend on the summation order."""
    return O.rnd(dt, rng.integers(-32, 33, size=(R, C)).astype(np.float32) / 8)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("hd", [128, 64])
@pytest.mark.parametrize("rope", [True, False])
@pytest.mark.parametrize("weights", [True, False])
def test_qk_norm_rope_exact_rows(pkg, dt, hd, rope, weights):
    rng = np.random.default_rng(hd + 2 * rope + weights)
    B, L, H, extra = 3, 40, 5, 48
    C = 3 * H * hd + extra
    x = exact_heads(rng, B * L, C, dt)
    qw = O.rnd(dt, rng.standard_normal(hd).astype(np.float32) * 0.3 + 1) if weights else None
    kw = O.rnd(dt, rng.standard_normal(hd).astype(np.float32) * 0.3 + 1) if weights else None
    cos, sin = rope_tables(L, hd) if rope else (None, None)
    t = dev(x, dt).view(B, L, C)
    pkg.ops.qk_norm_rope_(t, H, hd, None if qw is None else dev(qw, dt), None if kw is None else dev(kw, dt), 1e-6,
                          None if cos is None else torch.from_numpy(cos), None if sin is None else torch.from_numpy(sin))
    ref = O.qk_norm_rope(x, H, hd, dt, qw, kw, 1e-6, cos, sin, positions=L)
    np.testing.assert_array_equal(t.reshape(B * L, C).float().cpu().numpy(), ref)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_qk_norm_rope_strided_random(pkg, dt):
    """Rows of a wider buffer (a Flux single block's linear1 output: qkv then
    the MLP half), random values: within ``heads_close``, >= 99.9 %
    bit-equal; v and the MLP columns are untouched."""
    rng = np.random.default_rng(7)
    B, L, H, hd = 2, 520, 24, 128
    C = 3 * H * hd + 4 * H * hd
    x = O.rnd(dt, rng.standard_normal((B * L, C)).astype(np.float32) * 1.7)
    qw = O.rnd(dt, rng.standard_normal(hd).astype(np.float32) * 0.3 + 1)
    kw = O.rnd(dt, rng.standard_normal(hd).astype(np.float32) * 0.3 + 1)
    cos, sin = rope_tables(L, hd)
    full = dev(x, dt).view(B, L, C)
    view = full[..., :3 * H * hd]
    pkg.ops.qk_norm_rope_(view, H, hd, dev(qw, dt), dev(kw, dt), 1e-6, torch.from_numpy(cos), torch.from_numpy(sin))
    got = full.reshape(B * L, C).float().cpu().numpy()
    ref = O.qk_norm_rope(x, H, hd, dt, qw, kw, 1e-6, cos, sin, positions=L)
    assert heads_close(got, ref, H, hd, dt)
    assert (got != ref).mean() <= 1e-3
    np.testing.assert_array_equal(got[:, 2 * H * hd:], x[:, 2 * H * hd:])


def test_qk_norm_rope_matches_eager_torch(pkg):
    """Against the eager CUDA sequence it replaces (F.rms_norm, then the
    float32 rotary embedding), same tolerance."""
    torch.manual_seed(0)
    B, L, H, hd = 2, 300, 8, 128
    qkv = torch.randn((B, L, 3 * H * hd), device="cuda").to(torch.bfloat16)
    qn = (torch.randn(hd, device="cuda") * 0.2 + 1).to(torch.bfloat16)
    kn = (torch.randn(hd, device="cuda") * 0.2 + 1).to(torch.bfloat16)
    cos, sin = (torch.from_numpy(t).cuda() for t in rope_tables(L, hd))
    q, k, v = qkv.view(B, L, 3, H, hd).permute(2, 0, 3, 1, 4)

    def rope(x):
        a, b = x[..., 0::2].float(), x[..., 1::2].float()
        return torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1).flatten(-2).to(x.dtype)

    rq = rope(F.rms_norm(q, (hd,), qn, 1e-6)).float()
    rk = rope(F.rms_norm(k, (hd,), kn, 1e-6)).float()
    out = qkv.clone()
    pkg.ops.qk_norm_rope_(out, H, hd, qn, kn, 1e-6, cos, sin)
    gq, gk, gv = out.view(B, L, 3, H, hd).permute(2, 0, 3, 1, 4)
    for g, r in ((gq.float(), rq), (gk.float(), rk)):
        g2 = g.transpose(1, 2).reshape(B * L, H * hd).cpu().numpy()
        r2 = r.transpose(1, 2).reshape(B * L, H * hd).cpu().numpy()
        assert heads_close(np.concatenate([g2, g2], 1), np.concatenate([r2, r2], 1), H, hd, "bf16")
        assert (g != r).float().mean().item() <= 1e-3
    assert torch.equal(gv, v)
