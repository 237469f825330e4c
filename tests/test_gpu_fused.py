"""Parity of the fused DiT-step neighbours of the quantised linear (through
the C-ABI): the row norm + modulation prologue of the int8 activation
quantiser and the GELU / gated-residual epilogue of the W8A8 GEMM.

Bit parity with the oracle wherever the float32 arithmetic is fully
determined: rows whose statistics sum exactly in float32 (then the kernel's
summation order cannot matter) and the residual / gate steps.  Elsewhere the
tolerance is stated per test: the row statistics are summed in a different
(fixed) order than the oracle's float64 sums, and the oracle's numpy tanh is
not CUDA's tanhf, so a dtype rounding can flip by one unit.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import cuda_ok
from oracle import qlinear_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

TDT = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(scope="module")
def P(pkg):
    return pkg


def dev(a, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dt is not None:
        t = t.to(TDT[dt])
    return t.cuda()


def exact_rows(rng, M, K, dt, with_mean):
    """Rows of multiples of 1/8 in [-4, 4] whose sum is K*c exactly (c a
    multiple of 1/8, or 0): every float32 partial sum of the row, of
    (x - mean)^2 and of x^2 is exact, so the statistics do not depend on the
    summation order."""
    half = rng.integers(-24, 25, size=(M, K // 2)).astype(np.float32) / 8
    v = np.concatenate([half, -half], axis=1)
    v = np.take_along_axis(v, rng.permuted(np.tile(np.arange(K), (M, 1)), axis=1), axis=1)
    if with_mean:
        v = v + (rng.integers(-4, 5, size=(M, 1)).astype(np.float32) / 8)
    return O.rnd(dt, v)


def rnd_vec(rng, shape, dt, scale=1.0, offset=0.0):
    return O.rnd(dt, rng.standard_normal(shape).astype(np.float32) * scale + offset)


ROTS = [None, ("regular", 256), ("sylvester", 128)]


# ---------------------------------------------------------------------------
# prologue: norm + modulation + (rotation) + per-token int8
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("norm", ["layer", "rms"])
@pytest.mark.parametrize("rot", ROTS)
@pytest.mark.parametrize("M,K,S", [(37, 256, 1), (96, 3072, 3), (8, 4096, 2), (5, 1024, 5)])
def test_norm_quant_exact_rows(P, dt, norm, rot, M, K, S):
    rng = np.random.default_rng(M * 7 + K + S)
    x = exact_rows(rng, M, K, dt, with_mean=norm == "layer")
    w = rnd_vec(rng, K, dt, 0.5, 1.0) if norm == "rms" else None
    mul = O.rnd(dt, 1.0 + rnd_vec(rng, (S, K), dt, 0.3))
    add = rnd_vec(rng, (S, K), dt, 0.2)
    kw = dict(norm=norm, eps=1e-6, weight=w, mod_mul=mul, mod_add=add, rows_per_sample=M // S)
    q_ref, s_ref = O.norm_quant_int8(x, dt, rot, **kw)
    q, s = P.ops.quant_act_int8_norm(dev(x, dt), rot, norm=norm, eps=1e-6,
                                     norm_weight=None if w is None else dev(w, dt),
                                     mod_mul=dev(mul, dt), mod_add=dev(add, dt), rows_per_sample=M // S)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_ref.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("rot", [None, ("sylvester", 128)])
def test_norm_only_and_mod_only(P, dt, rot):
    """Each step on its own: norm without modulation, modulation without
    norm (multiply only, add only), single sample."""
    rng = np.random.default_rng(3)
    M, K = 64, 1024
    x = exact_rows(rng, M, K, dt, with_mean=True)
    mul = O.rnd(dt, 1.0 + rnd_vec(rng, K, dt, 0.3))
    add = rnd_vec(rng, K, dt, 0.2)
    cases = [dict(norm="layer"), dict(norm="rms"), dict(mod_mul=mul), dict(mod_add=add),
             dict(mod_mul=mul, mod_add=add)]
    for kw in cases:
        q_ref, s_ref = O.norm_quant_int8(x, dt, rot, **kw)
        args = {k: (dev(v, dt) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}
        q, s = P.ops.quant_act_int8_norm(dev(x, dt), rot, **args)
        np.testing.assert_array_equal(q.cpu().numpy(), q_ref, err_msg=str(list(kw)))
        np.testing.assert_array_equal(s.cpu().numpy(), s_ref, err_msg=str(list(kw)))


def _code_tolerance(q, q_ref, s, s_ref, max_frac):
    """Scales within one bf16 unit (the row absmax can move by one dtype
    unit); codes within one unit in rows with equal scales and within two
    where the scale moved (the code of an element that itself moved by one
    dtype unit is then also rescaled); at most ``max_frac`` codes differ."""
    np.testing.assert_allclose(s, s_ref, rtol=2.0 ** -7, atol=0)
    d = np.abs(q.astype(np.int32) - q_ref.astype(np.int32))
    same = (s.reshape(-1) == s_ref.reshape(-1))
    assert d[same].max(initial=0) <= 1
    assert d[~same].max(initial=0) <= 2
    assert d.astype(bool).mean() <= max_frac, d.astype(bool).mean()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("norm", ["layer", "rms"])
def test_norm_quant_dit_rows(P, dt, norm):
    """DiT-like activations (hidden 3072, two samples of 4608 tokens, Flux
    modulation) against the oracle and against the eager CUDA sequence the
    fused kernel replaces.  Tolerance: codes within 1 unit on <= 0.2% of
    elements against the oracle (a one-unit flip of a normalised value from
    the row statistics' summation order moves several rotated codes)."""
    rng = np.random.default_rng(11)
    S, L, K = 2, 4608, 3072
    M = S * L
    x = rnd_vec(rng, (M, K), dt, 1.5, 0.1)
    scale = rnd_vec(rng, (S, K), dt, 0.3)
    shift = rnd_vec(rng, (S, K), dt, 0.2)
    w = rnd_vec(rng, K, dt, 0.5, 1.0) if norm == "rms" else None
    rot = ("regular", 256)
    xt, sc, sh = dev(x, dt), dev(scale, dt), dev(shift, dt)
    mul_t = 1 + sc  # eager: (1 + scale) in the activation dtype
    q, s = P.ops.quant_act_int8_norm(xt, rot, norm=norm, eps=1e-6, norm_weight=None if w is None else dev(w, dt),
                                     mod_mul=mul_t, mod_add=sh, rows_per_sample=L)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    q_ref, s_ref = O.norm_quant_int8(x, dt, rot, norm=norm, eps=1e-6, weight=w, mod_mul=mul_t.float().cpu().numpy(),
                                     mod_add=shift, rows_per_sample=L)
    _code_tolerance(q, q_ref, s, s_ref, 2e-3)
    # the eager CUDA sequence: torch norm, broadcast modulation, then the
    # product quantiser
    x3 = xt.view(S, L, K)
    if norm == "layer":
        n = F.layer_norm(x3, (K,), eps=1e-6)
    else:
        n = F.rms_norm(x3, (K,), dev(w, dt), 1e-6)
    y = (n * mul_t[:, None] + sh[:, None]).reshape(M, K)
    qe, se = P.ops.quant_act_int8(y, rot)
    # torch's CUDA norms use their own statistics (Welford, rsqrtf): 0.5%
    _code_tolerance(q, qe.cpu().numpy(), s, se.cpu().numpy(), 5e-3)


def test_norm_quant_nonfinite_and_constant_rows(P):
    """A row holding Inf gives the quantiser's Inf/NaN row result (scale
    non-finite, codes 0); a constant row under layer norm is all zeros
    (scale clamps at 1e-30, codes 0), as in eager torch."""
    rng = np.random.default_rng(5)
    M, K = 8, 512
    x = rnd_vec(rng, (M, K), "bf16")
    x[2, 17] = np.inf
    x[5, :] = 0.75
    q, s = P.ops.quant_act_int8_norm(dev(x, "bf16"), None, norm="layer", eps=1e-6)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    assert not np.isfinite(s[2, 0]) and (q[2] == 0).all()
    assert s[5, 0] == np.float32(1e-30) and (q[5] == 0).all()
    keep = [r for r in range(M) if r not in (2, 5)]
    q_ref, s_ref = O.norm_quant_int8(x[keep], "bf16", None, norm="layer", eps=1e-6)
    _code_tolerance(q[keep], q_ref, s[keep], s_ref, 2e-3)


def test_norm_quant_empty_and_errors(P):
    x = torch.zeros((0, 256), dtype=torch.bfloat16, device="cuda")
    q, s = P.ops.quant_act_int8_norm(x, None, norm="layer")
    assert q.shape == (0, 256) and s.shape == (0, 1)
    x = torch.zeros((4, 256), dtype=torch.float32, device="cuda")
    with pytest.raises(TypeError):
        P.ops.quant_act_int8_norm(x, None, norm="layer")
    xb = x.to(torch.bfloat16)
    with pytest.raises(ValueError):
        P.ops.quant_act_int8_norm(xb, None, norm="group")
    with pytest.raises(ValueError):
        P.ops.quant_act_int8_norm(xb, None, mod_mul=torch.ones((3, 256), dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(P._native.NativeError):  # K % 16 != 0
        P.ops.quant_act_int8_norm(torch.zeros((4, 200), dtype=torch.bfloat16, device="cuda"), None, norm="rms")


# ---------------------------------------------------------------------------
# epilogue: GELU / residual + gate after the W8A8 epilogue
# ---------------------------------------------------------------------------


def _gemm_case(rng, M, N, K, dt):
    a = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    xs = (rng.random((M, 1), dtype=np.float32) * 0.02 + 1e-3).astype(np.float32)
    ws = (rng.random(N, dtype=np.float32) * 0.002 + 1e-4).astype(np.float32)
    b = rnd_vec(rng, N, dt, 0.5)
    return a, w, xs, ws, b


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K,G", [(512, 768, 256, 2), (300, 200, 512, 3), (100, 256, 128, 1), (4096, 3072, 3072, 2)])
@pytest.mark.parametrize("per_row", [True, False])
def test_gemm_residual_gate_exact(P, dt, M, N, K, G, per_row):
    rng = np.random.default_rng(M + N + K)
    a, w, xs, ws, b = _gemm_case(rng, M, N, K, dt)
    if not per_row:
        ws = ws[:1]
    res = rnd_vec(rng, (M, N), dt, 2.0)
    gate = rnd_vec(rng, (G, N), dt, 0.5)
    rpg = M // G
    Mg = rpg * G  # rows covered by whole gate groups
    acc = O.int_mm(a[:Mg], w)
    ep = O.w8a8_epilogue_per_row if per_row else O.w8a8_epilogue_tensorwise
    y_ref = ep(acc, xs[:Mg], ws if per_row else ws[0], b, dt)
    for g in (gate, None):
        ref = O.linear_post(y_ref, dt, residual=res[:Mg], gate=g, rows_per_gate=rpg)
        y = P.ops.gemm_w8a8_fused(dev(a[:Mg]), dev(xs[:Mg]), dev(w), dev(ws), dev(b, dt), TDT[dt], per_row=per_row,
                                  residual=dev(res[:Mg], dt), gate=None if g is None else dev(g, dt),
                                  rows_per_gate=rpg)
        np.testing.assert_array_equal(y.float().cpu().numpy(), ref)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K,gelu_from", [(512, 1024, 256, 0), (384, 1280, 512, 768), (64, 512, 256, 0),
                                             (4096, 12288, 3072, 0)])
def test_gemm_gelu(P, dt, M, N, K, gelu_from):
    """GELU in the epilogue against the exact function (the oracle, float64):
    one unit of the dtype relative, or 2^-20 absolute, on every output and
    a different value on <= 1% of them; against eager ``F.gelu(y,
    approximate="tanh")`` on the GPU within the same bound (its float32
    tanh form cancels below x = -3, where all values are under 2^-20)."""
    rng = np.random.default_rng(N + gelu_from)
    a, w, xs, ws, b = _gemm_case(rng, M, N, K, dt)
    y = P.ops.gemm_w8a8_fused(dev(a), dev(xs), dev(w), dev(ws), dev(b, dt), TDT[dt], gelu_from=gelu_from)
    plain = P.ops.gemm_w8a8(dev(a), dev(xs), dev(w), dev(ws), dev(b, dt), TDT[dt])
    unit = 2.0 ** -7 if dt == "bf16" else 2.0 ** -10
    eager = F.gelu(plain[:, gelu_from:], approximate="tanh").float()
    ge = y[:, gelu_from:].float()
    assert torch.all((ge - eager).abs() <= torch.clamp(eager.abs() * unit, min=2.0 ** -20))
    assert torch.equal(y[:, :gelu_from], plain[:, :gelu_from])
    ref = O.linear_post(plain.float().cpu().numpy(), dt, gelu_from=gelu_from)
    yo = y.float().cpu().numpy()
    np.testing.assert_array_equal(yo[:, :gelu_from], ref[:, :gelu_from])
    g, r = yo[:, gelu_from:], ref[:, gelu_from:]
    assert (np.abs(g - r) <= np.maximum(np.abs(r) * unit, 2.0 ** -20)).all()
    assert (g != r).mean() <= 0.01


def test_gemm_gelu_then_residual(P):
    """Both steps: residual + gate * gelu(y) (order of the epilogue), against
    the oracle with the exact GELU."""
    rng = np.random.default_rng(9)
    M, N, K = 512, 512, 256
    a, w, xs, ws, b = _gemm_case(rng, M, N, K, "bf16")
    res = rnd_vec(rng, (M, N), "bf16")
    gate = rnd_vec(rng, (2, N), "bf16", 0.5)
    y = P.ops.gemm_w8a8_fused(dev(a), dev(xs), dev(w), dev(ws), dev(b, "bf16"), torch.bfloat16, gelu_from=0,
                              residual=dev(res, "bf16"), gate=dev(gate, "bf16"))
    plain = P.ops.gemm_w8a8(dev(a), dev(xs), dev(w), dev(ws), dev(b, "bf16"), torch.bfloat16)
    ref = O.linear_post(plain.float().cpu().numpy(), "bf16", gelu_from=0, residual=res, gate=gate, rows_per_gate=M // 2)
    yo = y.float().cpu().numpy()
    # a GELU value one unit off moves gate * gelu by one unit of it, which
    # the residual add may round to one unit of the sum
    assert (np.abs(yo - ref) <= np.maximum(np.abs(ref), np.abs(res)) * 2.0 ** -7 + 2.0 ** -20).all()
    assert (yo != ref).mean() <= 0.01


def test_gemm_fused_strided_gate_and_errors(P):
    """A gate that is a column slice of a wider modulation output (row stride
    6N, as a Flux block's chunk(6) views) needs no copy; bad requests raise."""
    rng = np.random.default_rng(4)
    M, N, K = 256, 256, 128
    a, w, xs, ws, b = _gemm_case(rng, M, N, K, "bf16")
    mod = dev(rnd_vec(rng, (2, 6 * N), "bf16", 0.5), "bf16")
    gate = mod[:, 2 * N:3 * N]
    res = dev(rnd_vec(rng, (M, N), "bf16"), "bf16")
    y = P.ops.gemm_w8a8_fused(dev(a), dev(xs), dev(w), dev(ws), dev(b, "bf16"), torch.bfloat16, residual=res,
                              gate=gate)
    plain = P.ops.gemm_w8a8(dev(a), dev(xs), dev(w), dev(ws), dev(b, "bf16"), torch.bfloat16)
    assert torch.equal(y, res + torch.repeat_interleave(gate, M // 2, 0) * plain)
    with pytest.raises(ValueError):
        P.ops.gemm_w8a8_fused(dev(a), dev(xs), dev(w), dev(ws), None, torch.bfloat16, gate=gate)
    with pytest.raises(TypeError):
        P.ops.gemm_w8a8_fused(dev(a), dev(xs), dev(w), dev(ws), None, torch.float32, gelu_from=0)
    with pytest.raises(ValueError):
        P.ops.gemm_w8a8_fused(dev(a), dev(xs), dev(w), dev(ws), None, torch.bfloat16, residual=res[:100])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("B,Lt,Li,N,K", [(3, 128, 256, 512, 384), (2, 128, 640, 768, 256), (1, 256, 512, 256, 128)])
def test_gemm_segmented_rows(P, dt, B, Lt, Li, N, K):
    """Segmented rows (qlin_gemm_w8a8_fused_segments): the text / image
    streams of a joint [text | image] sequence of B samples.  Reading a
    stream's rows from the joint A and scales, or writing its output rows
    into the joint buffer, gives bit for bit the GEMM of the contiguous
    rows, with and without the gated residual; joint rows outside the
    written segments are untouched.  Odd sample counts leave a partial last
    pair tile (rows past M beyond the last segment)."""
    rng = np.random.default_rng(B * 1000 + Lt + Li)
    L = Lt + Li
    a, w, xs, ws, b = _gemm_case(rng, B * L, N, K, dt)
    A, XS, W, WS, BIAS = dev(a), dev(xs), dev(w), dev(ws), dev(b, dt)
    tdt = TDT[dt]
    parts = {"txt": (Lt, 0), "img": (Li, Lt)}

    def rows_of(t, n, off):  # the contiguous rows of one stream
        return t.view(B, L, *t.shape[1:])[:, off:off + n].reshape(B * n, *t.shape[1:]).contiguous()

    for name, (n, off) in parts.items():
        want = P.ops.gemm_w8a8(rows_of(A, n, off), rows_of(XS, n, off), W, WS, BIAS, tdt)
        got = P.ops.gemm_w8a8_fused(A, XS, W, WS, BIAS, tdt, a_rows=(n, L, off))
        assert torch.equal(got, want), name
        res = dev(rnd_vec(rng, (B * n, N), dt), dt)
        gate = dev(rnd_vec(rng, (B, N), dt, 0.5), dt)
        want_r = P.ops.gemm_w8a8_fused(rows_of(A, n, off), rows_of(XS, n, off), W, WS, BIAS, tdt, residual=res,
                                       gate=gate, rows_per_gate=n)
        got_r = P.ops.gemm_w8a8_fused(A, XS, W, WS, BIAS, tdt, a_rows=(n, L, off), residual=res, gate=gate,
                                      rows_per_gate=n)
        assert torch.equal(got_r, want_r), name
    # output segments: each stream's contiguous GEMM written into the joint rows
    joint = torch.full((B * L, N), 7.0, dtype=tdt, device="cuda")
    ref = joint.clone().view(B, L, N)
    for name, (n, off) in parts.items():
        xa, xsa = rows_of(A, n, off), rows_of(XS, n, off)
        out = P.ops.gemm_w8a8_fused(xa, xsa, W, WS, BIAS, tdt, out=joint, out_rows=(n, L, off))
        assert out.data_ptr() == joint.data_ptr()
        ref[:, off:off + n] = P.ops.gemm_w8a8(xa, xsa, W, WS, BIAS, tdt).view(B, n, N)
        assert torch.equal(joint, ref.view(B * L, N)), name  # the other stream's rows still hold 7.0 at first
    # both sides segmented in one call: the joint rows mapped onto themselves
    joint2 = torch.zeros_like(joint)
    for n, off in parts.values():
        P.ops.gemm_w8a8_fused(A, XS, W, WS, BIAS, tdt, a_rows=(n, L, off), out=joint2, out_rows=(n, L, off))
    assert torch.equal(joint2, P.ops.gemm_w8a8(A, XS, W, WS, BIAS, tdt))
    assert P.ops.device_error() == 0


def test_gemm_segmented_rows_errors(P):
    rng = np.random.default_rng(5)
    B, Lt, Li, N, K = 2, 128, 256, 256, 128
    L = Lt + Li
    a, w, xs, ws, b = _gemm_case(rng, B * L, N, K, "bf16")
    A, XS, W, WS = dev(a), dev(xs), dev(w), dev(ws)
    with pytest.raises(Exception):  # segments of 64 rows: not a multiple of 128
        P.ops.gemm_w8a8_fused(A, XS, W, WS, None, torch.bfloat16, a_rows=(64, L, 0))
    with pytest.raises(ValueError):  # the segment does not fit its stride
        P.ops.gemm_w8a8_fused(A, XS, W, WS, None, torch.bfloat16, a_rows=(256, L, 256))
    with pytest.raises(ValueError):  # out_rows without out
        P.ops.gemm_w8a8_fused(A, XS, W, WS, None, torch.bfloat16, out_rows=(Lt, L, 0))
    with pytest.raises(ValueError):  # M rows do not fill the output segments
        P.ops.gemm_w8a8_fused(A[:Lt * B], XS[:Lt * B], W, WS, None, torch.bfloat16,
                              out=torch.empty((3 * L, N), dtype=torch.bfloat16, device="cuda"), out_rows=(Lt, L, 0))
    with pytest.raises(Exception):  # 16 rows per output segment: not a multiple of 32
        P.ops.gemm_w8a8_fused(A[:512], XS[:512], W, WS, None, torch.bfloat16,
                              out=torch.empty((32 * 32, N), dtype=torch.bfloat16, device="cuda"), out_rows=(16, 32, 0))
    assert P.ops.device_error() == 0


# (img, txt) tokens: 96 / 32 take the torch.cat / slice path of the double
# blocks; 256 / 128 the segmented GEMM rows (128-row segments, 256 text rows)
@pytest.mark.parametrize("n_img,n_txt", [(96, 32), (256, 128)])
def test_dit_blocks_fused_match_unfused(P, monkeypatch, n_img, n_txt):
    """The measured DiT step with its neighbours fused (bench.py's
    dit_forward_fused: norm / modulation in the quantiser, GELU / residual in
    the GEMM epilogue, q/k norm + rotary kernel, concatenated linear2 input,
    segmented rows for the double blocks' joint sequence) against the same
    blocks with those steps eager around the plain quantised linear, on a
    small config: equal up to the norm statistics' order (relative L2 <=
    1e-2 after two double and two single blocks)."""
    import bench
    monkeypatch.setitem(bench.DIT, "hidden", 256)
    monkeypatch.setitem(bench.DIT, "heads", 2)
    monkeypatch.setitem(bench.DIT, "img", n_img)
    monkeypatch.setitem(bench.DIT, "txt", n_txt)
    dev_ = torch.device("cuda", 0)
    rot = (bench.DIT["kind"], bench.DIT["group"])
    params = bench._dit_params(dev_, lambda w: P.ops.quant_weight_int8(w, rot), 2, 2)
    lin, fl = bench.dit_linears(P, rot)

    img, txt, vec = bench.dit_inputs(2, dev_, 7)
    with torch.no_grad():
        a = bench.dit_forward_fused(params, img, txt, vec, fl, P.ops.qk_norm_rope_).float()
        b = bench.dit_forward(params, img, txt, vec, lin).float()
    assert torch.isfinite(a).all()
    assert ((a - b).norm() / b.norm()).item() <= 1e-2


# ---------------------------------------------------------------------------
# SiTU prologue of the activation quantiser (qlin_quant_act_int8_situ)
# ---------------------------------------------------------------------------

SITU_ROTS = [None, ("regular", 256), ("sylvester", 128), ("regular", 16)]


def situ_rows(rng, M, K, pad, dt):
    x = rng.standard_normal((M, 2 * K + pad)).astype(np.float32) * 3
    x[0, :8] = 1e-3              # the small-|x| tanh branch
    x[-1, K:K + 8] = -40.0        # sigmoid(gate) underflows towards 0
    return x


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("rot", SITU_ROTS)
@pytest.mark.parametrize("M,K,pad", [(37, 3072, 0), (5, 256, 64), (130, 1024, 16), (3, 12288, 0), (64, 512, 0)])
def test_situ_quant_matches_two_calls(P, dt, rot, M, K, pad):
    """Bit-equal to ops.situ followed by ops.quant_act_int8 (the same
    device SiTU function, then the same rotation and quantisation); rows
    read in place from a wider buffer when pad > 0."""
    if rot is not None and K % rot[1]:
        pytest.skip("row length not a multiple of the rotation block")
    rng = np.random.default_rng(M + K + pad)
    full = dev(situ_rows(rng, M, K, pad, dt), dt)
    x = full[:, :2 * K]
    q, s = P.ops.quant_act_int8_situ(x, rot)
    q_ref, s_ref = P.ops.quant_act_int8(P.ops.situ(x), rot)
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref)
    assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    assert P.ops.device_error() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_situ_quant_vs_float64(P, dt):
    """Against a float64 SiTU rounded once to the dtype, then the oracle's
    quantisation: scales within one dtype unit of the row maximum / 127,
    codes within one step."""
    rng = np.random.default_rng(11)
    M, K = 48, 1024
    x = O.rnd(dt, situ_rows(rng, M, K, 0, dt))
    q, s = P.ops.quant_act_int8_situ(dev(x, dt), None)
    x64 = x.astype(np.float64)
    h, g = x64[:, :K], x64[:, K:]
    y = O.rnd(dt, (4 * np.tanh(g / 4) / (1 + np.exp(-g)) * 25 * np.tanh(h / 25)).astype(np.float32))
    qo, so = O.quantize_int8_axiswise(y, dim=-1)
    sg = s.cpu().numpy().reshape(-1)
    unit = 2.0 ** (-7 if dt == "bf16" else -10)
    assert np.all(np.abs(sg - so.reshape(-1)) <= unit * so.reshape(-1) + 1e-30)
    assert np.abs(q.cpu().numpy().astype(np.int32) - qo.astype(np.int32)).max() <= 1


def test_situ_quant_errors(P):
    x = torch.zeros((4, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        P.ops.quant_act_int8_situ(x.float(), None)   # float32 rows: not taken by the prologue
    with pytest.raises(ValueError):
        P.ops.quant_act_int8_situ(x[:, :63], None)   # odd row: no [hidden | gate] split
    st = torch.cuda.current_stream().cuda_stream
    q = torch.empty((4, 24), dtype=torch.int8, device="cuda")
    s = torch.empty((4,), dtype=torch.float32, device="cuda")
    with pytest.raises(P._native.NativeError):      # K = 24: not a multiple of 16
        P._native.call("qlin_quant_act_int8_situ", x.data_ptr(), 0, 4, 24, 64, 0, 0, 0.0, q.data_ptr(),
                       s.data_ptr(), st)
    with pytest.raises(P._native.NativeError):      # ldx < 2K
        P._native.call("qlin_quant_act_int8_situ", x.data_ptr(), 0, 4, 48, 64, 0, 0, 0.0, q.data_ptr(),
                       s.data_ptr(), st)
    q0, s0 = P.ops.quant_act_int8_situ(x[:0], None)
    assert q0.shape == (0, 32) and s0.shape == (0, 1)


@pytest.mark.parametrize("convrot", [False, True])
def test_kitchen_int8_linear_situ_fused(P, convrot):
    """kitchen_patch.int8_linear with input_act="situ": the fused quantiser
    path equals the two-call path (situ, then the linear without it)."""
    kp = P.kitchen_patch
    rng = np.random.default_rng(5)
    B, L, K, N = 2, 40, 1024, 384
    x = dev(rng.standard_normal((B, L, 2 * K)).astype(np.float32) * 2, "bf16")
    w = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32) * 0.02).cuda()
    rot = P.int8_quant.rot_for_group(256) if convrot else None
    wq, ws = P.ops.quant_weight_int8(w, rot)
    b = dev(rng.standard_normal(N).astype(np.float32) * 0.1, "bf16")
    y = kp.int8_linear(x, wq, ws, b, torch.bfloat16, convrot=convrot, convrot_groupsize=256, input_act="situ")
    y_ref = kp.int8_linear(P.ops.situ(x), wq, ws, b, torch.bfloat16, convrot=convrot, convrot_groupsize=256)
    assert y.shape == (B, L, N)
    assert torch.equal(y, y_ref)
