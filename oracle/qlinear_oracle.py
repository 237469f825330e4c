"""CPU oracle for the quantized-linear hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the PyTorch CPU path of the ComfyUI INT8-Fast
node pack (v1.3.4) for the functions on the quantized-linear hot path.  It is
the checker that the CUDA kernels are compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it; the product path never does.

Parity pinning: every function below that restates a reference function is
checked against golden vectors produced by running the reference's own code
(``tests/golden/make_golden.py`` imports it with stub ``comfy`` modules) in
``tests/test_oracle_golden.py``.  Functions marked RESTATEMENT cover schemes
that do not exist in the reference (group-128 int4); they follow the
reference's int4 conventions and are pinned only by the self-consistency
properties tested there.

Value conventions
-----------------
Activations are carried as float32 arrays whose values are exactly
representable in the compute dtype ("bf16", "f16" or "f32"); ``rnd(dtype, v)``
rounds a float32 array to that dtype (round-to-nearest-even) and returns it as
float32 again.  All float arithmetic is float32 with one IEEE rounding per
operation, exactly like torch's CPU kernels for these element-wise ops.
Integer matrix products use float64 BLAS, which is exact here because every
partial sum stays below 2**53.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32

# ---------------------------------------------------------------------------
# dtype rounding helpers
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round-to-nearest-even (c10::BFloat16)."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = r.copy()
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def rnd(dtype: str, v) -> np.ndarray:
    """Round float32 values to ``dtype`` and return them as float32."""
    v = np.asarray(v, dtype=F32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(v)).reshape(v.shape)
    if dtype == "f16":
        return v.astype(np.float16).astype(F32)
    if dtype == "f32":
        return v
    raise ValueError(dtype)


def fp8_e4m3fn_to_f32(b: np.ndarray) -> np.ndarray:
    """Decode float8_e4m3fn bytes (bias 7, no inf, 0x7f/0xff = NaN)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int32)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    normal = s * (1.0 + m / 8.0) * np.exp2(e - 7.0)
    sub = s * (m / 8.0) * 2.0 ** -6
    out = np.where(e == 0, sub, normal)
    out = np.where((b & 0x7F) == 0x7F, np.nan, out)
    return out.astype(F32)


# ---------------------------------------------------------------------------
# INT8 quantizers -- int8_quant.py:41-55
# ---------------------------------------------------------------------------


def quantize_int8(x: np.ndarray, scale) -> np.ndarray:
    """int8_quant.py:41-42: ``x.float().mul(1.0 / scale).round_().clamp_(-128, 127)``.

    ``1.0 / scale`` on a tensor is ``scale.reciprocal() * 1.0`` (an IEEE
    float32 division), the multiply is float32 RN and ``round_`` is
    round-half-even."""
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        inv = F32(1.0) / np.asarray(scale, dtype=F32)
        q = np.rint(np.asarray(x, dtype=F32) * inv)
    # a NaN product (Inf/NaN rows) casts to int8 code 0, as torch's cast does
    q = np.where(np.isnan(q), 0, q)
    return np.clip(q, -128, 127).astype(np.int8)


def quantize_int8_axiswise(x: np.ndarray, dim: int):
    """int8_quant.py:49-52: per-axis absmax/127 (clamped at 1e-30) int8 quant.

    Returns (q int8, scale float32 with ``dim`` kept as size 1)."""
    x = np.asarray(x, dtype=F32)
    amax = np.abs(x).max(axis=dim, keepdims=True)
    scale = np.maximum(amax / F32(127.0), F32(1e-30)).astype(F32)
    return quantize_int8(x, scale), scale


def quantize_int8_tensorwise(x: np.ndarray):
    """int8_quant.py:44-47."""
    x = np.asarray(x, dtype=F32)
    scale = np.maximum(np.abs(x).max() / F32(127.0), F32(1e-30)).astype(F32)
    return quantize_int8(x, scale), scale


def dequantize(q: np.ndarray, scale) -> np.ndarray:
    """int8_quant.py:54-55."""
    return q.astype(F32) * np.asarray(scale, dtype=F32)


# ---------------------------------------------------------------------------
# Integer GEMM -- torch._int_mm / triton_int4_mm semantics
# ---------------------------------------------------------------------------


def int_mm(a: np.ndarray, b_nk: np.ndarray) -> np.ndarray:
    """``torch._int_mm(a, b.T)``: int8 [M,K] x int8 [N,K]^T -> int32 [M,N].

    float64 BLAS is exact: |partial sum| <= K*128*128 < 2**53."""
    a = np.asarray(a)
    b = np.asarray(b_nk)
    assert a.shape[1] == b.shape[1]
    return (a.astype(np.float64) @ b.astype(np.float64).T).astype(np.int32)


# ---------------------------------------------------------------------------
# W8A8 forward -- int8_quant.py:113-164 (CPU branch)
# ---------------------------------------------------------------------------


def w8a8_epilogue_per_row(acc, x_scale, w_scale, bias, dtype):
    """int8_quant.py:158-163:
    ``res.float().mul_(x_scale).mul_(weight_scale.T).to(dtype)`` then
    ``+ bias.to(dtype)`` (a dtype add: float32 add, one more rounding)."""
    r = acc.astype(F32)
    r = r * np.asarray(x_scale, F32).reshape(-1, 1)
    r = r * np.asarray(w_scale, F32).reshape(1, -1)
    y = rnd(dtype, r)
    if bias is not None:
        y = rnd(dtype, y + rnd(dtype, np.asarray(bias, F32)).reshape(1, -1))
    return y


def w8a8_epilogue_tensorwise(acc, x_scale, w_scale, bias, dtype):
    """int8_quant.py:129-133: ``res.float().mul_(weight_scale * x_scale)``."""
    s = (F32(np.asarray(w_scale, F32).reshape(())) * np.asarray(x_scale, F32).reshape(-1, 1)).astype(F32)
    y = rnd(dtype, acc.astype(F32) * s)
    if bias is not None:
        y = rnd(dtype, y + rnd(dtype, np.asarray(bias, F32)).reshape(1, -1))
    return y


def int8_forward_dynamic_per_row(x, w_q, w_scale, bias, dtype):
    """int8_quant.py:137-164, CPU branch (the parity target)."""
    xq, xs = quantize_int8_axiswise(x, dim=-1)
    acc = int_mm(xq, w_q)
    return w8a8_epilogue_per_row(acc, xs, w_scale, bias, dtype)


def int8_forward_dynamic(x, w_q, w_scale, bias, dtype):
    """int8_quant.py:113-133, CPU branch (scalar weight scale)."""
    xq, xs = quantize_int8_axiswise(x, dim=-1)
    acc = int_mm(xq, w_q)
    return w8a8_epilogue_tensorwise(acc, xs, w_scale, bias, dtype)


# ---------------------------------------------------------------------------
# ConvRot Hadamard -- convrot.py:18-118
# ---------------------------------------------------------------------------

_H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.int64)


def hadamard_int(size: int, kind: str) -> np.ndarray:
    """Integer (+-1) Hadamard matrix.

    kind "regular": convrot.py:36-52, H4 of Theorem 3.3 Kronecker-powered
    (``torch.kron(H, H4)``); size must be a power of 4.
    kind "sylvester": ``scipy.linalg.hadamard`` (imported at convrot.py:12),
    the only construction that exists for sizes that are not powers of 4."""
    if kind == "regular":
        if size < 4 or size & (size - 1) or (size.bit_length() - 1) % 2:
            raise ValueError(f"Regular Hadamard size must be a power of 4, got {size}")
        h = _H4
        while h.shape[0] < size:
            h = np.kron(h, _H4)
        return h
    if kind == "sylvester":
        if size < 2 or size & (size - 1):
            raise ValueError(f"Sylvester Hadamard size must be a power of 2, got {size}")
        h = np.array([[1]], dtype=np.int64)
        while h.shape[0] < size:
            h = np.block([[h, h], [h, -h]])
        return h
    raise ValueError(kind)


def hadamard_scale(size: int, dtype: str) -> float:
    """The +-entry of the normalised matrix as used by the rotation:
    ``H / size**0.5`` built in float32 (convrot.py:54), then cast to the
    activation dtype (``H.to(dtype=x.dtype)``, convrot.py:116)."""
    # torch: H_int(float32) / (size ** 0.5): the double scalar is cast to
    # float32 and the +-1 entries divided by it in float32.
    c = F32(np.float32(1.0) / np.float32(size ** 0.5))
    return float(rnd(dtype, c))


def _digit_radix4_regular(v: np.ndarray, stride: int) -> np.ndarray:
    """One base-4 digit of the regular H4 transform, in the fixed float32 order
    that the CUDA kernels use: S = (a0+a1)+(a2+a3); y_k = S - 2*a_{3-k}."""
    n = v.shape[-1]
    w = v.reshape(v.shape[:-1] + (n // (4 * stride), 4, stride))
    a0, a1, a2, a3 = (w[..., i, :] for i in range(4))
    s = (a0 + a1) + (a2 + a3)
    y = np.stack([s - F32(2) * a3, s - F32(2) * a2, s - F32(2) * a1, s - F32(2) * a0], axis=-2)
    return y.reshape(v.shape).astype(F32)


def _digit_radix2_sylvester(v: np.ndarray, stride: int) -> np.ndarray:
    n = v.shape[-1]
    w = v.reshape(v.shape[:-1] + (n // (2 * stride), 2, stride))
    a0, a1 = w[..., 0, :], w[..., 1, :]
    y = np.stack([a0 + a1, a0 - a1], axis=-2)
    return y.reshape(v.shape).astype(F32)


def hadamard_transform_f32(x: np.ndarray, group: int, kind: str) -> np.ndarray:
    """Unnormalised block Hadamard transform of the last axis, in groups of
    ``group``, evaluated digit by digit from the least significant index digit
    upwards in float32 (the order the CUDA kernels use).  Mathematically this
    is ``x.view(..., K/g, g) @ H_int`` of convrot.py:114-117."""
    x = np.asarray(x, dtype=F32)
    K = x.shape[-1]
    if K % group:
        raise ValueError(f"features {K} not divisible by group_size {group}")
    v = x.reshape(x.shape[:-1] + (K // group, group)).copy()
    stride = 1
    if kind == "regular":
        hadamard_int(group, "regular")
        while stride < group:
            v = _digit_radix4_regular(v, stride)
            stride *= 4
    elif kind == "sylvester":
        hadamard_int(group, "sylvester")
        while stride < group:
            v = _digit_radix2_sylvester(v, stride)
            stride *= 2
    else:
        raise ValueError(kind)
    return v.reshape(x.shape)


def rotate(x: np.ndarray, group: int, kind: str, dtype: str) -> np.ndarray:
    """``rotate_activation`` (convrot.py:89-118) / ``rotate_weight``
    (convrot.py:58-86; H is symmetric so W @ H^T == W @ H): the fixed-order
    float32 transform times the dtype-rounded normalisation constant, rounded
    to ``dtype``.

    The reference evaluates the same sum with a library matmul whose float32
    accumulation order is unspecified; the two agree to 1 unit in the last
    place of ``dtype`` (pinned against the reference in the golden tests)."""
    c = F32(hadamard_scale(group, dtype))
    return rnd(dtype, hadamard_transform_f32(x, group, kind) * c)


def rotate_exact(x: np.ndarray, group: int, kind: str, dtype: str) -> np.ndarray:
    """Correctly rounded rotation (float64 sum, one rounding) -- used only by
    tests to bound the float32-order error of ``rotate``."""
    h = hadamard_int(group, kind).astype(np.float64)
    c = float(hadamard_scale(group, dtype))
    K = x.shape[-1]
    v = np.asarray(x, np.float64).reshape(x.shape[:-1] + (K // group, group)) @ h
    v = (v * c).reshape(x.shape)
    # float64 -> float32 -> dtype may double-round in rare ties; tests only
    # use this as an error bound, never for bit comparisons.
    return rnd(dtype, v.astype(F32))


# ---------------------------------------------------------------------------
# INT4 -- int4_quant.py:36-134, 292-353
# ---------------------------------------------------------------------------

INT4_MAX = 7


def pack_int4_row_major(values: np.ndarray) -> np.ndarray:
    """int4_quant.py:36-47: low nibble = even K column, high = odd."""
    v = np.asarray(values)
    if v.shape[-1] % 2:
        raise ValueError(f"last dim must be even, got {v.shape[-1]}")
    lo = v[..., 0::2].astype(np.int32) & 0x0F
    hi = v[..., 1::2].astype(np.int32) & 0x0F
    return (lo | (hi << 4)).astype(np.uint8).view(np.int8)


def unpack_int4_row_major(packed: np.ndarray) -> np.ndarray:
    """int4_quant.py:50-58 (signed nibbles)."""
    p = np.asarray(packed).astype(np.int32) & 0xFF
    lo = p & 0x0F
    hi = (p >> 4) & 0x0F
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return np.stack([lo, hi], axis=-1).reshape(p.shape[:-1] + (-1,)).astype(np.int8)


def int4_clamp_min(dtype: str) -> float:
    """``clamp(min=1e-10)`` on a ``dtype`` tensor compares against 1e-10
    converted to that dtype."""
    return float(rnd(dtype, F32(1e-10)))


def quantize_signed_int4(x: np.ndarray, dtype: str, axis: int = -1):
    """int4_quant.py:65-73 / 76-83: all in ``dtype``:
    absmax.clamp(1e-10) -> scale = absmax / 7 -> (x / scale).round().clamp(+-7).

    Returns (q int8 in [-7, 7], scale float32 with ``axis`` kept)."""
    x = np.asarray(x, dtype=F32)
    amax = np.abs(x).max(axis=axis, keepdims=True)
    amax = np.maximum(amax, F32(int4_clamp_min(dtype)))
    s = rnd(dtype, amax / F32(INT4_MAX))
    with np.errstate(invalid="ignore", divide="ignore"):
        q = np.rint(rnd(dtype, x / s))
    # an all-zero f16 row divides 0/0 (the 1e-10 clamp underflows in f16);
    # torch casts the NaN to int8 code 0
    q = np.where(np.isnan(q), 0, q)
    return np.clip(q, -INT4_MAX, INT4_MAX).astype(np.int8), s.astype(F32)


def quantize_signed_int4_rowwise(x, dtype):
    q, s = quantize_signed_int4(x, dtype)
    return q, s.reshape(-1)


def quantize_signed_int4_rowwise_packed(x, dtype):
    q, s = quantize_signed_int4(x, dtype)
    return pack_int4_row_major(q), s.reshape(-1)


def quantize_signed_int4_grouped(x, dtype, group=128):
    """RESTATEMENT (not in the reference): the int4_quant.py:65-73 conventions
    applied per contiguous group of ``group`` along K.  Returns
    (q int8 [R,K], scales float32 [R, K/group])."""
    x = np.asarray(x, dtype=F32)
    R, K = x.shape
    if K % group:
        raise ValueError("K % group")
    q, s = quantize_signed_int4(x.reshape(R, K // group, group), dtype, axis=-1)
    return q.reshape(R, K), s.reshape(R, K // group)


def w4a4_rowwise_epilogue(acc, x_scale, w_scale, bias, dtype):
    """int4_quant.py:338-353: float32 ``acc * x_scale * w_scale (+ bias)``,
    rounded once to ``dtype``."""
    out = acc.astype(F32) * np.asarray(x_scale, F32).reshape(-1, 1)
    out = out * np.asarray(w_scale, F32).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, F32).reshape(1, -1)
    return rnd(dtype, out)


def convrot_w4a4_forward(x, w_packed, w_scale, bias, group, kind, dtype, skip_rotation=False):
    """int4_quant.py:292-353 with ``triton_int4_mm`` replaced by its defined
    semantics (triton_int4_mm.py:4-9): ``a @ unpack(W).T`` in int32."""
    xr = x if skip_rotation else rotate(x, group, kind, dtype)
    qa, sa = quantize_signed_int4_rowwise(xr, dtype)
    acc = int_mm(qa, unpack_int4_row_major(w_packed))
    return w4a4_rowwise_epilogue(acc, sa, w_scale, bias, dtype)


def quantize_convrot_w4a4_weight(w, group, kind, dtype="f32"):
    """int4_quant.py:121-134 (weight in float32 at load time)."""
    wr = rotate(w, group, kind, dtype)
    return quantize_signed_int4_rowwise_packed(wr, dtype)


# --- group-128 schemes (RESTATEMENT, not in the reference) -----------------


def fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Correctly rounded float32 fused multiply-add a*b+c (IEEE fmaf).

    a*b is exact in float64 for the operands used here (|a| < 2**24 integers
    times bf16-representable b); the float64 sum is then corrected with an
    error-free TwoSum so that ties at float32 rounding boundaries are broken
    by the exact residual."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    c = np.asarray(c, np.float64)
    p = a * b
    s = p + c
    bp = s - c
    err = (p - bp) + (c - (s - bp))  # TwoSum residual: p + c == s + err exactly
    r = s.astype(F32)
    # float64 -> float32 rounding of s; if s sits exactly on a float32
    # midpoint, the true value is on the side of err.
    r64 = r.astype(np.float64)
    up = np.nextafter(r, np.float32(np.inf)).astype(np.float64)
    dn = np.nextafter(r, np.float32(-np.inf)).astype(np.float64)
    tie_hi = (s == (r64 + up) / 2)
    tie_lo = (s == (r64 + dn) / 2)
    r = np.where(tie_hi & (err > 0), np.nextafter(r, np.float32(np.inf)), r)
    r = np.where(tie_lo & (err < 0), np.nextafter(r, np.float32(-np.inf)), r)
    return r.astype(F32)


def group_partials(a_q: np.ndarray, w_q: np.ndarray, group: int = 128) -> np.ndarray:
    """int32 partial dot products per K-group: [G, M, N]."""
    M, K = a_q.shape
    G = K // group
    out = np.empty((G, M, w_q.shape[0]), dtype=np.int32)
    for g in range(G):
        sl = slice(g * group, (g + 1) * group)
        out[g] = int_mm(a_q[:, sl], w_q[:, sl])
    return out


def w4a8_g128_forward_from_q(a_q, a_scale, w_packed, w_gscale, bias, dtype, group=128):
    """RESTATEMENT for packed-INT4 W4A8 with per-group weight scales:
    acc = 0; for g: acc = fmaf(float(P_g), ws[n, g], acc);
    y = dtype(acc * xs[m] + bias) (int4_quant.py:338-353 style, one rounding)."""
    w_q = unpack_int4_row_major(w_packed)
    P = group_partials(a_q, w_q, group)
    ws = np.asarray(w_gscale, F32)
    acc = np.zeros(P.shape[1:], dtype=F32)
    for g in range(P.shape[0]):
        acc = fma_f32(P[g].astype(F32), ws[:, g].reshape(1, -1), acc)
    out = acc * np.asarray(a_scale, F32).reshape(-1, 1)
    if bias is not None:
        out = out + np.asarray(bias, F32).reshape(1, -1)
    return rnd(dtype, out)


def w4a4_g128_forward_from_q(a_q, a_gscale, w_packed, w_gscale, bias, dtype, group=128):
    """RESTATEMENT for W4A4 with per-group scales on both operands:
    acc = fmaf(float(P_g), xs[m,g] * ws[n,g], acc) over g; y = dtype(acc + bias)."""
    w_q = unpack_int4_row_major(w_packed)
    P = group_partials(a_q, w_q, group)
    xs = np.asarray(a_gscale, F32)
    ws = np.asarray(w_gscale, F32)
    acc = np.zeros(P.shape[1:], dtype=F32)
    for g in range(P.shape[0]):
        s = (xs[:, g].reshape(-1, 1) * ws[:, g].reshape(1, -1)).astype(F32)
        acc = fma_f32(P[g].astype(F32), s, acc)
    out = acc
    if bias is not None:
        out = out + np.asarray(bias, F32).reshape(1, -1)
    return rnd(dtype, out)


# ---------------------------------------------------------------------------
# Asymmetric W4A8 (Lloyd-Max codebook) -- w4a8_int8.py:29-75 + int8_quant.py:679-687
# ---------------------------------------------------------------------------


def unpack_int4_unsigned(packed: np.ndarray) -> np.ndarray:
    """w4a8_int8.py:29-43."""
    p = np.asarray(packed).astype(np.int32) & 0xFF
    return np.stack([p & 0x0F, (p >> 4) & 0x0F], axis=-1).reshape(p.shape[:-1] + (-1,))


def dequant_asym_w4a8_to_float(packed, codebook, s_channel, s_rel_fp8, group_size):
    """w4a8_int8.py:46-75: codebook[code] * s_channel[n] * s_rel[n, k // gs]."""
    codes = unpack_int4_unsigned(packed)
    N, K = codes.shape
    vals = np.asarray(codebook, F32)[codes]
    s_rel = fp8_e4m3fn_to_f32(s_rel_fp8)
    if s_rel.shape[1] * group_size != K:
        raise ValueError("W4A8: group mismatch")
    s_rel_x = np.repeat(s_rel, group_size, axis=1)
    return ((vals * np.asarray(s_channel, F32).reshape(N, 1)) * s_rel_x).astype(F32)


def requant_asym_w4a8(packed, codebook, s_channel, s_rel_fp8, group_size):
    """int8_quant.py:679-687: dequant then ``quantize_int8_axiswise(dim=1)``."""
    return quantize_int8_axiswise(dequant_asym_w4a8_to_float(packed, codebook, s_channel, s_rel_fp8, group_size), dim=1)


# ---------------------------------------------------------------------------
# Weight-side helpers for loaders and LoRA -- int8_quant.py:517-554, 809-843
# ---------------------------------------------------------------------------


def quantize_weight_int8(w, group=0, kind="regular"):
    """OTF weight quant (int8_quant.py:527-554): float32 weight, optional
    ConvRot ``rotate_weight``, then ``quantize_int8_axiswise(dim=1)``."""
    w = np.asarray(w, F32)
    if group:
        w = rotate(w, group, kind, "f32")
    return quantize_int8_axiswise(w, dim=1)


def dequant_unrotate_int8(q, scale, group=0, kind="regular"):
    """LoRA bake, steps 1-2 (int8_quant.py:815-825 / 909-918):
    ``dequantize`` then ``rotate_weight`` (H is its own inverse)."""
    w = dequantize(q, np.asarray(scale, F32).reshape(-1, 1) if np.size(scale) > 1 else scale)
    if group:
        w = rotate(w, group, kind, "f32")
    return w


def rotate_requant_int8(w, scale, group=0, kind="regular"):
    """LoRA bake, steps 4-5 (int8_quant.py:830-843 / 925-941):
    ``rotate_weight`` then ``quantize_int8`` with the ORIGINAL scale."""
    w = np.asarray(w, F32)
    if group:
        w = rotate(w, group, kind, "f32")
    s = np.asarray(scale, F32)
    s = s.reshape(-1, 1) if s.size > 1 else s.reshape(())
    return quantize_int8(w, s)


# ---------------------------------------------------------------------------
# Neighbours of the linear in a DiT block -- the eager PyTorch sequence that
# the fused prologue / epilogue replace (kitchen input_act and residual form,
# rocm_int8_kitchen_patch.py:136, 176; a Flux block's LayerNorm + modulation
# in front of Int8TensorwiseOps.Linear, int8_quant.py:633-716, and its gated
# residual / GELU behind it).  RESTATEMENT of torch's element-wise rounding:
# every eager op rounds to the activation dtype.  Row statistics are summed in
# float64 and rounded once, so they are exact whenever the float32 sums are
# (the kernels sum in float32 in their own fixed order; eager torch in its
# own) -- tests use exactly summable rows for bit parity and a tolerance
# elsewhere.
# ---------------------------------------------------------------------------

GELU_BETA = F32(0.7978845608028654)  # sqrt(2 / pi)
GELU_KAPPA = F32(0.044715)


def rsqrt_rn(v: np.ndarray) -> np.ndarray:
    """float32 1/sqrt(v) (float64 evaluation, one rounding to float32)."""
    return (1.0 / np.sqrt(np.asarray(v, np.float64))).astype(F32)


def row_norm(x: np.ndarray, kind: str, eps: float, dtype: str, weight=None) -> np.ndarray:
    """``F.layer_norm(x, (K,), eps=eps)`` (no affine; kind "layer") or
    ``F.rms_norm(x, (K,), weight, eps)`` (kind "rms": ``dt((x * rstd) *
    weight)``, one rounding) on rows of ``dtype`` values."""
    x = np.asarray(x, F32)
    K = F32(x.shape[-1])
    e = F32(eps)
    if kind == "layer":
        mean = (x.astype(np.float64).sum(-1, keepdims=True).astype(F32) / K).astype(F32)
        d = (x - mean).astype(F32)
        var = ((d.astype(np.float64) ** 2).sum(-1, keepdims=True).astype(F32) / K).astype(F32)
        rstd = rsqrt_rn((var + e).astype(F32))
        return rnd(dtype, d * rstd)
    if kind == "rms":
        ms = ((x.astype(np.float64) ** 2).sum(-1, keepdims=True).astype(F32) / K).astype(F32)
        rstd = rsqrt_rn((ms + e).astype(F32))
        y = (x * rstd).astype(F32)
        if weight is not None:
            y = (y * np.asarray(weight, F32)).astype(F32)
        return rnd(dtype, y)
    raise ValueError(kind)


def _per_sample(v, M: int, rows_per: int) -> np.ndarray:
    """[S, N] (or [N]) per-sample rows broadcast to the M rows of x."""
    v = np.asarray(v, F32)
    if v.ndim == 1:
        v = v[None, :]
    return v[np.arange(M) // rows_per]


def norm_modulate(x, dtype: str, norm=None, eps: float = 1e-6, weight=None, mod_mul=None, mod_add=None,
                  rows_per_sample=None) -> np.ndarray:
    """``dt(norm(x))``, ``dt(. * mod_mul[s])``, ``dt(. + mod_add[s])`` (a Flux
    block's ``layer_norm(x) * (1 + scale) + shift`` with ``mod_mul = dt(1 +
    scale)``), sample ``s = row // rows_per_sample``."""
    y = np.asarray(x, F32)
    M = y.shape[0]
    rps = rows_per_sample or M
    if norm is not None:
        y = row_norm(y, norm, eps, dtype, weight)
    if mod_mul is not None:
        y = rnd(dtype, y * _per_sample(mod_mul, M, rps))
    if mod_add is not None:
        y = rnd(dtype, y + _per_sample(mod_add, M, rps))
    return y


def norm_quant_int8(x, dtype: str, rot=None, **kw):
    """Fused prologue + per-token int8: (q, scale[M, 1])."""
    y = norm_modulate(x, dtype, **kw)
    if rot is not None:
        y = rotate(y, rot[1], rot[0], dtype)
    return quantize_int8_axiswise(y, dim=-1)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """The tanh-form GELU ``0.5 x (1 + tanh(u))``, ``u = sqrt(2/pi) (x +
    0.044715 x^3)`` (``F.gelu(approximate="tanh")``), evaluated exactly in
    float64 as the equal ``x / (1 + exp(-2u))`` and rounded once to float32.
    Kernels are held within one unit of the 16-bit dtype of this value;
    eager PyTorch's float32 tanh form differs from it by more where
    ``1 + tanh(u)`` cancels (x < -3, values below 2^-20 there)."""
    x64 = np.asarray(x, F32).astype(np.float64)
    u = np.sqrt(2.0 / np.pi) * (x64 + 0.044715 * x64 ** 3)
    with np.errstate(over="ignore", invalid="ignore"):
        y = x64 / (1.0 + np.exp(-2.0 * u))
    return y.astype(F32)


def linear_post(y, dtype: str, gelu_from=None, residual=None, gate=None, rows_per_gate=None) -> np.ndarray:
    """The element-wise steps after a quantised linear's output ``y`` (dtype
    values): ``dt(gelu_tanh(y))`` on columns ``>= gelu_from``, then
    ``dt(residual + dt(gate[g] * y))`` (or ``dt(residual + y)``)."""
    y = np.array(y, F32)
    M = y.shape[0]
    if gelu_from is not None:
        y[:, gelu_from:] = rnd(dtype, gelu_tanh(y[:, gelu_from:]))
    if residual is not None:
        t = y if gate is None else rnd(dtype, _per_sample(gate, M, rows_per_gate or M) * y)
        y = rnd(dtype, np.asarray(residual, F32) + t)
    return y


def qk_norm_rope(qkv, heads: int, head_dim: int, dtype: str, q_weight=None, k_weight=None, eps: float = 1e-6,
                 cos=None, sin=None, positions=None) -> np.ndarray:
    """The attention prologue of a Flux-style DiT block on rows ``qkv`` [R, C]
    (C >= 3*heads*head_dim; q heads, k heads, v heads): every q and k head
    vector gets ``F.rms_norm(x, (head_dim,), weight, eps)`` (``row_norm``
    "rms") and then the rotary embedding of adjacent pairs in float32,
    ``(c*a - s*b, s*a + c*b)`` with every product and sum rounded to float32
    and the result rounded once to ``dtype`` (Flux's apply_rope on float32
    tables ``cos`` / ``sin`` [positions, head_dim/2], table row = row %
    positions).  Returns a new array; v and the columns after it are kept.
    No counterpart in the reference (ComfyUI's model code)."""
    x = np.array(qkv, F32, copy=True)
    R = x.shape[0]
    D = heads * head_dim
    for part, w in ((0, q_weight), (1, k_weight)):
        v = x[:, part * D:(part + 1) * D].reshape(R * heads, head_dim)
        n = row_norm(v, "rms", eps, dtype, w).reshape(R, heads, head_dim)
        if cos is not None:
            pos = np.arange(R) % (positions or R)
            c = np.asarray(cos, F32)[pos][:, None, :]
            s = np.asarray(sin, F32)[pos][:, None, :]
            a, b = n[..., 0::2], n[..., 1::2]
            o0 = ((c * a).astype(F32) - (s * b).astype(F32)).astype(F32)
            o1 = ((s * a).astype(F32) + (c * b).astype(F32)).astype(F32)
            n = rnd(dtype, np.stack((o0, o1), axis=-1).reshape(R, heads, head_dim))
        x[:, part * D:(part + 1) * D] = n.reshape(R, D)
    return x
