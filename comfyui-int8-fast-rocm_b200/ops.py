"""Torch-facing wrappers of the sm_100a kernels.

Each function validates/normalises its tensors, allocates the outputs with
``torch.empty`` on the input's device, and calls one C-ABI entry point of
libqlinear_b200 on torch's current CUDA stream.  CUDA tensors only: there is
no CPU path (a CPU tensor raises).
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _native as N

_DT = {torch.bfloat16: N.BF16, torch.float16: N.F16, torch.float32: N.F32}
_ROT = {None: N.ROT_NONE, "none": N.ROT_NONE, "regular": N.ROT_REGULAR, "sylvester": N.ROT_SYLVESTER}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    if not t.is_cuda:
        raise RuntimeError(
            "comfyui-int8-fast-rocm_b200 kernels run on CUDA (sm_100a) tensors only; got a tensor on " + str(t.device))
    N.call("qlin_set_device", t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous with a 16-byte aligned base (copies only when needed)."""
    if not t.is_contiguous():
        t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _rows(x: torch.Tensor):
    """2-D view with unit inner stride; returns (x2d, ldx)."""
    if x.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(x.shape)}")
    if x.stride(1) != 1 or x.stride(0) < x.shape[1]:
        x = x.contiguous()
    return x, x.stride(0)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected bfloat16, float16 or float32") from None


def hadamard_scale(group: int, dtype: torch.dtype) -> float:
    """The +-entry of the normalised Hadamard ``H / group**0.5`` (built in
    float32, convrot.py:54) after the cast to the operand dtype
    (``H.to(dtype=x.dtype)``, convrot.py:116)."""
    c = torch.ones((), dtype=torch.float32) / (group ** 0.5)
    return float(c.to(dtype).float().item())


def _rot_args(rot, dtype):
    """rot: None or (kind, group) with kind in {"regular", "sylvester"}."""
    if rot is None:
        return N.ROT_NONE, 0, 0.0
    kind, group = rot
    return _ROT[kind], int(group), hadamard_scale(int(group), dtype)


def int4_clamp_min(dtype: torch.dtype) -> float:
    """``clamp(min=1e-10)`` on a ``dtype`` tensor (int4_quant.py:70)."""
    return float(torch.tensor(1e-10, dtype=dtype).float().item())


# ---------------------------------------------------------------------------
# (a) activations
# ---------------------------------------------------------------------------


def quant_act_int8(x: torch.Tensor, rot=None):
    """Per-token int8: (q int8 [M,K], scale float32 [M,1])."""
    x, ldx = _rows(x)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    if M and K:
        st = _stream(x)
        kind, g, c = _rot_args(rot, x.dtype)
        if kind != N.ROT_NONE and x.data_ptr() % 16:
            x, ldx = x.clone(), K
        N.call("qlin_quant_act_int8", x.data_ptr(), dtype_code(x.dtype), M, K, ldx, kind, g, c,
               q.data_ptr(), s.data_ptr(), st)
    return q, s


_NORM = {None: N.NORM_NONE, "none": N.NORM_NONE, "layer": N.NORM_LAYER, "layer_norm": N.NORM_LAYER,
         "rms": N.NORM_RMS, "rms_norm": N.NORM_RMS}


def _vec_rows(v: torch.Tensor, K: int, dtype: torch.dtype, device):
    """A per-sample parameter ([K] or [S, K], unit inner stride) as
    (tensor, row stride); copies only when the layout does not fit."""
    if v.dim() == 1:
        v = v.reshape(1, -1)
    if v.dim() != 2 or v.shape[1] != K:
        raise ValueError(f"expected a [K] or [S, K] tensor with K={K}, got shape {tuple(v.shape)}")
    if v.dtype != dtype or v.device != device:
        v = v.to(device=device, dtype=dtype)
    fits = v.stride(1) == 1 and v.data_ptr() % 16 == 0 and (v.stride(0) * v.element_size()) % 16 == 0 and \
        (v.shape[0] == 1 or v.stride(0) >= K)
    if not fits:
        v = _aligned(v)
    return v, (v.stride(0) if v.shape[0] > 1 else K)


def quant_act_int8_norm(x: torch.Tensor, rot=None, norm=None, eps: float = 1e-6, norm_weight=None, mod_mul=None,
                        mod_add=None, rows_per_sample=None):
    """Per-token int8 of a DiT block's normalised, modulated activation:
    ``y = dt(norm(x))``, ``y = dt(y * mod_mul[s])``, ``y = dt(y + mod_add[s])``
    (sample ``s = row // rows_per_sample``), then the rotation and the
    quantisation of :func:`quant_act_int8`, in one pass over ``x``.

    ``norm``: None, ``"layer"`` (F.layer_norm without affine) or ``"rms"``
    (F.rms_norm with ``norm_weight``); ``mod_mul`` / ``mod_add``: ``[K]`` or
    ``[S, K]`` in x.dtype (bf16 / f16).  Returns (q int8 [M,K], scale [M,1])."""
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"the fused norm prologue takes bfloat16 or float16 input, got {x.dtype}")
    if norm not in _NORM:
        raise ValueError(f"norm must be one of {sorted(k for k in _NORM if k)} or None, got {norm!r}")
    x, ldx = _rows(x)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    if M == 0 or K == 0:
        return q, s
    st = _stream(x)
    if x.data_ptr() % 16:
        x, ldx = x.clone(), K
    kind, g, c = _rot_args(rot, x.dtype)
    w = None
    if norm_weight is not None:
        w, _ = _vec_rows(norm_weight.reshape(-1), K, x.dtype, x.device)
    mm = ma = None
    mul_ld = add_ld = K
    if mod_mul is not None:
        mm, mul_ld = _vec_rows(mod_mul, K, x.dtype, x.device)
    if mod_add is not None:
        ma, add_ld = _vec_rows(mod_add, K, x.dtype, x.device)
    S = max([t.shape[0] for t in (mm, ma) if t is not None] or [1])
    rps = int(rows_per_sample) if rows_per_sample is not None else (M // S if S > 1 else M)
    if rows_per_sample is None and S > 1 and rps * S != M:
        raise ValueError(f"{M} rows do not split into {S} samples")
    if rps <= 0 or -(-M // rps) > S:  # every row's sample must have a modulation row
        raise ValueError(f"rows_per_sample={rps} needs {-(-M // max(rps, 1))} modulation rows, got {S}")
    N.call("qlin_quant_act_int8_norm", x.data_ptr(), dtype_code(x.dtype), M, K, ldx, _NORM[norm], float(eps),
           _ptr(w), _ptr(mm), mul_ld, _ptr(ma), add_ld, rps, kind, g, c, q.data_ptr(), s.data_ptr(), st)
    return q, s


def quant_act_int8_cat(x1: torch.Tensor, x2: torch.Tensor, rot=None):
    """Per-token int8 of the row concatenation ``torch.cat((x1, x2), -1)``
    without materialising it: ``x1`` [M, K1] and ``x2`` [M, K2] (row-strided
    views are read in place, e.g. column slices of a wider output).  Returns
    (q int8 [M, K1 + K2], scale float32 [M, 1])."""
    if x1.dim() != 2 or x2.dim() != 2 or x1.shape[0] != x2.shape[0]:
        raise ValueError(f"expected [M, K1] and [M, K2] tensors, got {tuple(x1.shape)} and {tuple(x2.shape)}")
    if x1.dtype != x2.dtype or x1.device != x2.device:
        raise ValueError("the two parts must share dtype and device")
    x1, ld1 = _rows(x1)
    x2, ld2 = _rows(x2)
    M, K1 = x1.shape
    K2 = x2.shape[1]
    q = torch.empty((M, K1 + K2), dtype=torch.int8, device=x1.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x1.device)
    if M == 0:
        return q, s
    st = _stream(x1)
    es = x1.element_size()
    if x1.data_ptr() % 16 or (ld1 * es) % 16:
        x1, ld1 = x1.contiguous().clone(), K1
    if x2.data_ptr() % 16 or (ld2 * es) % 16:
        x2, ld2 = x2.contiguous().clone(), K2
    kind, g, c = _rot_args(rot, x1.dtype)
    N.call("qlin_quant_act_int8_cat", x1.data_ptr(), ld1, K1, x2.data_ptr(), ld2, K2, dtype_code(x1.dtype), M,
           kind, g, c, q.data_ptr(), s.data_ptr(), st)
    return q, s


def quant_act_int8_situ(x: torch.Tensor, rot=None):
    """Per-token int8 of ``situ(x)`` for ``x`` [M, 2K] = [hidden | gate]
    (bf16/f16, K % 16 == 0; row-strided views are read in place) without
    writing the [M, K] activation: bit-equal to
    ``quant_act_int8(situ(x), rot)``.  Returns (q int8 [M, K], scale
    float32 [M, 1])."""
    if x.dim() != 2 or x.shape[1] % 2:
        raise ValueError(f"expected [M, 2K] rows ([hidden | gate]), got {tuple(x.shape)}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"the SiTU prologue takes bf16 or f16 input, got {x.dtype}")
    x2, ldx = _rows(x)
    M, K = x2.shape[0], x2.shape[1] // 2
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    if M == 0 or K == 0:
        return q, s
    if x2.data_ptr() % 16 or (ldx * x2.element_size()) % 16:
        x2, ldx = x2.contiguous().clone(), 2 * K
    kind, g, c = _rot_args(rot, x.dtype)
    N.call("qlin_quant_act_int8_situ", x2.data_ptr(), dtype_code(x.dtype), M, K, ldx, kind, g, c, q.data_ptr(),
           s.data_ptr(), _stream(x2))
    return q, s


def qk_norm_rope_(qkv: torch.Tensor, heads: int, head_dim: int, q_weight=None, k_weight=None, eps: float = 1e-6,
                  cos=None, sin=None) -> torch.Tensor:
    """In place on the fused qkv projection ``qkv`` [..., L, >= 3*heads*head_dim]
    (bf16/f16, unit inner stride, rows may be strided): every q and k head
    vector becomes ``rope(dt(F.rms_norm(x, (head_dim,), weight, eps)))``;
    ``cos`` / ``sin`` are float32 [L, head_dim // 2] tables indexed by the
    token position within its sample (None: no rotation); the rotation of
    the pair (a, b) = (n[2i], n[2i+1]) is (c*a - s*b, s*a + c*b), each float32
    product and sum rounded, then rounded to the dtype.  Returns ``qkv``."""
    if qkv.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"qk_norm_rope_ takes bfloat16 or float16, got {qkv.dtype}")
    if qkv.stride(-1) != 1:
        raise ValueError("qkv needs a unit inner stride")
    ld = qkv.stride(-2) if qkv.dim() >= 2 else qkv.shape[-1]
    rows = qkv.numel() // qkv.shape[-1]
    if qkv.dim() >= 3:  # rows must be evenly strided across the leading dims
        for d in range(qkv.dim() - 2):
            if qkv.stride(d) != qkv.stride(d + 1) * qkv.shape[d + 1]:
                raise ValueError("qkv rows must be evenly strided")
    positions = qkv.shape[-2] if qkv.dim() >= 2 else 1
    st = _stream(qkv)

    def vec(w):
        if w is None:
            return None
        w = w.reshape(-1).to(device=qkv.device, dtype=qkv.dtype)
        if w.numel() != head_dim:
            raise ValueError(f"norm weight must have {head_dim} elements")
        return _aligned(w)

    qw, kw = vec(q_weight), vec(k_weight)
    ct = stb = None
    if cos is not None:
        ct = _aligned(cos.to(device=qkv.device, dtype=torch.float32).reshape(positions, head_dim // 2))
        stb = _aligned(sin.to(device=qkv.device, dtype=torch.float32).reshape(positions, head_dim // 2))
    N.call("qlin_qk_norm_rope", qkv.data_ptr(), dtype_code(qkv.dtype), rows, ld, int(heads), int(head_dim),
           _ptr(qw), _ptr(kw), float(eps), _ptr(ct), _ptr(stb), positions, st)
    return qkv


def quant_act_int4(x: torch.Tensor, rot=None, group: int = 0):
    """Signed int4-range codes in int8 storage: (q [M,K], scale float32
    [M] (group 0) or [M, K/128] (group 128))."""
    x, ldx = _rows(x)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,) if group == 0 else (M, K // 128), dtype=torch.float32, device=x.device)
    if M and K:
        st = _stream(x)
        kind, g, c = _rot_args(rot, x.dtype)
        if (kind != N.ROT_NONE or group) and x.data_ptr() % 16:
            x, ldx = x.clone(), K
        N.call("qlin_quant_act_int4", x.data_ptr(), dtype_code(x.dtype), M, K, ldx, kind, g, c, int(group),
               int4_clamp_min(x.dtype), q.data_ptr(), s.data_ptr(), st)
    return q, s


def rotate(x: torch.Tensor, kind: str, group: int) -> torch.Tensor:
    """Block-diagonal Hadamard rotation of the last dim (rotate_activation /
    rotate_weight semantics), result in x.dtype."""
    shape = x.shape
    x2, ldx = _rows(x.reshape(-1, shape[-1]))
    M, K = x2.shape
    out = torch.empty((M, K), dtype=x.dtype, device=x.device)
    if M and K:
        st = _stream(x2)
        if x2.data_ptr() % 16:
            x2, ldx = x2.clone(), K
        k, g, c = _rot_args((kind, group), x.dtype)
        N.call("qlin_rotate", x2.data_ptr(), dtype_code(x.dtype), M, K, ldx, k, g, c, out.data_ptr(), st)
    return out.reshape(shape)


def situ(x: torch.Tensor) -> torch.Tensor:
    """[..., 2K] ([hidden | gate]) -> [..., K] SiTU activation in x.dtype."""
    k2 = x.shape[-1]
    if k2 % 2:
        raise ValueError(f"situ expects an even last dim ([hidden | gate]), got {k2}")
    K = k2 // 2
    x2, ldx = _rows(x.reshape(-1, k2))
    M = x2.shape[0]
    y = torch.empty((M, K), dtype=x.dtype, device=x.device)
    if M and K:
        st = _stream(x2)
        N.call("qlin_situ", x2.data_ptr(), dtype_code(x.dtype), M, K, ldx, y.data_ptr(), st)
    return y.reshape(*x.shape[:-1], K)


# ---------------------------------------------------------------------------
# (b) / (c) GEMMs
# ---------------------------------------------------------------------------


def _check_gemm(a, w, k_factor=1):
    if a.dtype != torch.int8 or w.dtype != torch.int8:
        raise TypeError("int8 operands expected")
    if a.dim() != 2 or w.dim() != 2:
        raise ValueError("2-D operands expected")
    if a.shape[1] != w.shape[1] * k_factor:
        raise ValueError(f"K mismatch: activation K={a.shape[1]}, weight represents {w.shape[1] * k_factor}")
    if a.device != w.device:
        raise ValueError("operands on different devices")


def _pad_k(a_q, w, mult, w_factor=1):
    """Zero-pad K to a multiple of ``mult`` (zero columns add nothing to the
    int32 sums)."""
    K = a_q.shape[1]
    if K % mult:
        pad = mult - K % mult
        a_q = F.pad(a_q, (0, pad))
        w = F.pad(w, (0, pad // w_factor))
    return a_q, w


# Split-K scratch of the W8A8 GEMM: bytes per (device, M, N, K), and one
# zero-initialised buffer per (device, stream) -- calls on one stream run in
# order, and every complete call leaves the buffer's counters at zero.
_SPLITK_BYTES = {}
_SPLITK_SCRATCH = {}


def _splitk_scratch(device, M, Nn, K, stream):
    key = (device.index, M, Nn, K)
    nbytes = _SPLITK_BYTES.get(key)
    if nbytes is None:
        out = ctypes.c_uint64(0)
        N.call("qlin_gemm_w8a8_splitk_scratch", M, Nn, K, ctypes.addressof(out))
        nbytes = _SPLITK_BYTES[key] = int(out.value)
    if nbytes == 0:
        return None
    skey = (device.index, stream)
    buf = _SPLITK_SCRATCH.get(skey)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _SPLITK_SCRATCH[skey] = buf
    return buf


def gemm_w8a8(a_q, a_scale, w_q, w_scale, bias=None, out_dtype=torch.bfloat16, per_row=True):
    """W8A8 linear on int8 operands (int8_forward_dynamic(_per_row) epilogue).
    Problems too small to fill the GPU with 256 x 256 tiles split K over CTA
    pairs (``qlin_gemm_w8a8_splitk``, same output bits)."""
    _check_gemm(a_q, w_q)
    a_q, w_q = _pad_k(_aligned(a_q), _aligned(w_q), 16)
    M, K = a_q.shape
    Nn = w_q.shape[0]
    out = torch.empty((M, Nn), dtype=out_dtype, device=a_q.device)
    if M == 0 or Nn == 0:
        return out
    a_scale = a_scale.reshape(-1).to(device=a_q.device, dtype=torch.float32).contiguous()
    w_scale = w_scale.reshape(-1).to(device=a_q.device, dtype=torch.float32).contiguous()
    if per_row and w_scale.numel() != Nn:
        raise ValueError(f"per-row weight scale must have {Nn} entries, got {w_scale.numel()}")
    if not per_row and w_scale.numel() != 1:
        raise ValueError("tensorwise weight scale must be a scalar")
    if bias is not None:
        bias = bias.reshape(-1).to(device=a_q.device, dtype=out_dtype).contiguous()
    st = _stream(a_q)
    scratch = _splitk_scratch(a_q.device, M, Nn, K, st)
    if scratch is not None:
        N.call("qlin_gemm_w8a8_splitk", a_q.data_ptr(), a_scale.data_ptr(), w_q.data_ptr(), w_scale.data_ptr(),
               N.WSCALE_ROW if per_row else N.WSCALE_TENSOR, _ptr(bias), out.data_ptr(), dtype_code(out_dtype),
               M, Nn, K, scratch.data_ptr(), scratch.numel(), st)
        return out
    N.call("qlin_gemm_w8a8", a_q.data_ptr(), a_scale.data_ptr(), w_q.data_ptr(), w_scale.data_ptr(),
           N.WSCALE_ROW if per_row else N.WSCALE_TENSOR, _ptr(bias), out.data_ptr(), dtype_code(out_dtype),
           M, Nn, K, st)
    return out


def _segments(rows, total, what):
    n, stride, off = (int(v) for v in rows)
    if n <= 0 or stride < n or off < 0 or off + n > stride:
        raise ValueError(f"{what}: segments of {n} rows at {off} of every {stride} do not fit")
    if total % stride:
        raise ValueError(f"{what}: {total} rows are not whole strides of {stride}")
    return n, stride, off


def gemm_w8a8_fused(a_q, a_scale, w_q, w_scale, bias=None, out_dtype=torch.bfloat16, per_row=True, gelu_from=None,
                    residual=None, gate=None, rows_per_gate=None, a_rows=None, out=None, out_rows=None):
    """:func:`gemm_w8a8` with a DiT block's element-wise steps in the
    epilogue: ``y = dt(gelu_tanh(y))`` for output columns ``>= gelu_from``,
    then ``y = dt(residual + dt(gate[g] * y))`` (``dt(residual + y)`` without
    ``gate``), gate row ``g = row // rows_per_gate``.  ``residual`` [M, N],
    ``gate`` [N] or [G, N], both cast to ``out_dtype`` (bf16 / f16).

    Segmented rows (CTA-pair kernel, M and N >= 256): ``a_rows=(n, stride,
    off)`` takes the linear's logical rows from ``a_q`` / ``a_scale`` as the
    n rows at offset ``off`` of every ``stride`` rows (M = a_q rows //
    stride * n; n a multiple of 128); ``out_rows=(n, stride, off)`` writes
    them into ``out`` ([R, N] contiguous, R a multiple of stride) the same
    way (n a multiple of 32), and ``out`` is returned.  A Flux double
    block's text and image streams use this to write q/k/v into the joint
    sequence and to read their projections' rows from the joint attention
    output without torch.cat or slice copies."""
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"the fused epilogue writes bfloat16 or float16, got {out_dtype}")
    _check_gemm(a_q, w_q)
    a_q, w_q = _pad_k(_aligned(a_q), _aligned(w_q), 16)
    R, K = a_q.shape
    Nn = w_q.shape[0]
    aseg = oseg = (0, 0, 0)
    M = R
    if a_rows is not None:
        aseg = _segments(a_rows, R, "a_rows")
        M = R // aseg[1] * aseg[0]
    if out_rows is not None:
        if out is None:
            raise ValueError("out_rows needs out")
        if out.dtype != out_dtype or out.dim() != 2 or out.shape[1] != Nn or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [R, {Nn}] {out_dtype} tensor")
        oseg = _segments(out_rows, out.shape[0], "out_rows")
        if M % oseg[0] or M // oseg[0] != out.shape[0] // oseg[1]:
            raise ValueError(f"{M} rows do not fill the {out.shape[0] // oseg[1]} output segments of {oseg[0]}")
    elif out is not None:
        if tuple(out.shape) != (M, Nn) or out.dtype != out_dtype or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [{M}, {Nn}] {out_dtype} tensor")
    else:
        out = torch.empty((M, Nn), dtype=out_dtype, device=a_q.device)
    if M == 0 or Nn == 0:
        return out
    a_scale = a_scale.reshape(-1).to(device=a_q.device, dtype=torch.float32).contiguous()
    if a_scale.numel() != R:
        raise ValueError(f"a_scale must have {R} entries, got {a_scale.numel()}")
    w_scale = w_scale.reshape(-1).to(device=a_q.device, dtype=torch.float32).contiguous()
    if per_row and w_scale.numel() != Nn:
        raise ValueError(f"per-row weight scale must have {Nn} entries, got {w_scale.numel()}")
    if not per_row and w_scale.numel() != 1:
        raise ValueError("tensorwise weight scale must be a scalar")
    if bias is not None:
        bias = bias.reshape(-1).to(device=a_q.device, dtype=out_dtype).contiguous()
    gelu_col0 = Nn if gelu_from is None else max(0, int(gelu_from))
    ld_res = gate_ld = Nn
    rpg = M
    if residual is not None:
        if tuple(residual.shape) != (M, Nn):
            raise ValueError(f"residual must be [{M}, {Nn}], got {tuple(residual.shape)}")
        residual, ld_res = _vec_rows(residual, Nn, out_dtype, a_q.device)
        if residual.shape[0] == 1:
            ld_res = Nn
    if gate is not None:
        if residual is None:
            raise ValueError("a gate needs a residual")
        gate, gate_ld = _vec_rows(gate, Nn, out_dtype, a_q.device)
        G = gate.shape[0]
        rpg = int(rows_per_gate) if rows_per_gate is not None else M // G
        if rows_per_gate is None and rpg * G != M:
            raise ValueError(f"{M} rows do not split into {G} gate rows")
        if rpg <= 0 or -(-M // rpg) > G:  # every row's gate row must exist
            raise ValueError(f"rows_per_gate={rpg} needs {-(-M // max(rpg, 1))} gate rows, got {G}")
    st = _stream(a_q)
    if aseg[0] or oseg[0]:
        N.call("qlin_gemm_w8a8_fused_segments", a_q.data_ptr(), a_scale.data_ptr(), w_q.data_ptr(),
               w_scale.data_ptr(), N.WSCALE_ROW if per_row else N.WSCALE_TENSOR, _ptr(bias), out.data_ptr(),
               dtype_code(out_dtype), M, Nn, K, gelu_col0, _ptr(residual), ld_res, _ptr(gate), gate_ld, rpg,
               *aseg, *oseg, st)
        return out
    N.call("qlin_gemm_w8a8_fused", a_q.data_ptr(), a_scale.data_ptr(), w_q.data_ptr(), w_scale.data_ptr(),
           N.WSCALE_ROW if per_row else N.WSCALE_TENSOR, _ptr(bias), out.data_ptr(), dtype_code(out_dtype),
           M, Nn, K, gelu_col0, _ptr(residual), ld_res, _ptr(gate), gate_ld, rpg, st)
    return out


def int_mm(a_q, w_q):
    """int32 [M,N] = a_q [M,K] . w_q[N,K]^T (``torch._int_mm(a, w.T)``)."""
    _check_gemm(a_q, w_q)
    a_q, w_q = _pad_k(_aligned(a_q), _aligned(w_q), 16)
    M, K = a_q.shape
    Nn = w_q.shape[0]
    c = torch.empty((M, Nn), dtype=torch.int32, device=a_q.device)
    if M == 0 or Nn == 0:
        return c
    if K == 0:
        return c.zero_()
    st = _stream(a_q)
    N.call("qlin_int_mm", a_q.data_ptr(), w_q.data_ptr(), c.data_ptr(), M, Nn, K, st)
    return c


def int4_mm(a_q, w_packed):
    """int32 [M,N] = a_q [M,K] . unpack(w_packed [N,K/2])^T (triton_int4_mm)."""
    _check_gemm(a_q, w_packed, 2)
    a_q, w_packed = _pad_k(_aligned(a_q), _aligned(w_packed), 32, 2)
    M, K = a_q.shape
    Nn = w_packed.shape[0]
    c = torch.empty((M, Nn), dtype=torch.int32, device=a_q.device)
    if M == 0 or Nn == 0:
        return c
    st = _stream(a_q)
    N.call("qlin_int4_mm", a_q.data_ptr(), w_packed.data_ptr(), c.data_ptr(), M, Nn, K, st)
    return c


def gemm_w4a4(a_q, a_scale, w_packed, w_scale, bias=None, out_dtype=torch.bfloat16):
    """W4A4 per-row linear with the convrot_w4a4_forward epilogue."""
    _check_gemm(a_q, w_packed, 2)
    a_q, w_packed = _pad_k(_aligned(a_q), _aligned(w_packed), 32, 2)
    M, K = a_q.shape
    Nn = w_packed.shape[0]
    out = torch.empty((M, Nn), dtype=out_dtype, device=a_q.device)
    if M == 0 or Nn == 0:
        return out
    a_scale = a_scale.reshape(-1).to(device=a_q.device, dtype=torch.float32).contiguous()
    w_scale = w_scale.reshape(-1).to(device=a_q.device, dtype=torch.float32).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(device=a_q.device, dtype=out_dtype).contiguous()
    st = _stream(a_q)
    N.call("qlin_gemm_w4a4", a_q.data_ptr(), a_scale.data_ptr(), w_packed.data_ptr(), w_scale.data_ptr(),
           _ptr(bias), out.data_ptr(), dtype_code(out_dtype), M, Nn, K, st)
    return out


def gemm_w4_g128(a_q, a_scale, w_packed, w_gscale, bias=None, out_dtype=torch.bfloat16, a_int4_groups=False):
    """Group-128 W4A8 (a_scale [M]) or W4A4 (a_scale [M, K/128]) linear;
    w_gscale [N, K/128] (bf16 values)."""
    _check_gemm(a_q, w_packed, 2)
    a_q, w_packed = _aligned(a_q), _aligned(w_packed)
    M, K = a_q.shape
    Nn = w_packed.shape[0]
    out = torch.empty((M, Nn), dtype=out_dtype, device=a_q.device)
    if M == 0 or Nn == 0:
        return out
    a_scale = a_scale.to(device=a_q.device, dtype=torch.float32).contiguous()
    ws = w_gscale.to(device=a_q.device, dtype=torch.bfloat16).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(device=a_q.device, dtype=out_dtype).contiguous()
    st = _stream(a_q)
    fn = "qlin_gemm_w4a4_g128" if a_int4_groups else "qlin_gemm_w4a8_g128"
    N.call(fn, a_q.data_ptr(), a_scale.data_ptr(), w_packed.data_ptr(), ws.data_ptr(), _ptr(bias),
           out.data_ptr(), dtype_code(out_dtype), M, Nn, K, st)
    return out


# ---------------------------------------------------------------------------
# (d) weights
# ---------------------------------------------------------------------------


def quant_weight_int8(w: torch.Tensor, rot=None):
    """w [N,K] (bf16/f16/f32) -> .float() -> optional rotate_weight ->
    quantize_int8_axiswise(dim=1): (q int8 [N,K], scale float32 [N,1])."""
    w = _aligned(w)
    Nn, K = w.shape
    q = torch.empty((Nn, K), dtype=torch.int8, device=w.device)
    s = torch.empty((Nn, 1), dtype=torch.float32, device=w.device)
    if Nn and K:
        st = _stream(w)
        kind, g, c = _rot_args(rot, torch.float32)
        N.call("qlin_quant_weight_int8", w.data_ptr(), dtype_code(w.dtype), Nn, K, kind, g, c, q.data_ptr(),
               s.data_ptr(), st)
    return q, s


def quant_weight_int4(w: torch.Tensor, rot=None, group: int = 0):
    """Packed signed int4 [N,K/2] + scales: float32 [N] (group 0, float32
    math as quantize_convrot_w4a4_weight) or [N, K/128] (group 128, math in
    w.dtype)."""
    w = _aligned(w)
    Nn, K = w.shape
    p = torch.empty((Nn, K // 2), dtype=torch.int8, device=w.device)
    s = torch.empty((Nn,) if group == 0 else (Nn, K // 128), dtype=torch.float32, device=w.device)
    if Nn and K:
        st = _stream(w)
        kind, g, c = _rot_args(rot, torch.float32 if group == 0 else w.dtype)
        N.call("qlin_quant_weight_int4", w.data_ptr(), dtype_code(w.dtype), Nn, K, kind, g, c, int(group),
               p.data_ptr(), s.data_ptr(), st)
    return p, s


def requant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size: int):
    """asym_w4a8_int8 -> int8 per-channel (q [N,K], scale float32 [N,1])."""
    packed = _aligned(packed)
    Nn, Kp = packed.shape
    K = Kp * 2
    dev = packed.device
    codebook = codebook.to(device=dev, dtype=torch.float32).contiguous()
    s_channel = s_channel.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    if s_rel.dtype != torch.uint8:
        s_rel = s_rel.view(torch.uint8)
    s_rel = s_rel.to(dev).contiguous()
    if s_rel.shape[1] * group_size != K:
        raise ValueError(f"W4A8: group mismatch, num_groups({s_rel.shape[1]}) * group_size({group_size}) != K({K})")
    q = torch.empty((Nn, K), dtype=torch.int8, device=dev)
    s = torch.empty((Nn, 1), dtype=torch.float32, device=dev)
    if Nn and K:
        st = _stream(packed)
        N.call("qlin_requant_asym_w4a8", packed.data_ptr(), codebook.data_ptr(), s_channel.data_ptr(),
               s_rel.data_ptr(), int(group_size), Nn, K, q.data_ptr(), s.data_ptr(), st)
    return q, s


def dequant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size: int) -> torch.Tensor:
    """asym_w4a8_int8 -> float32 [N, K]: codebook[code] * s_channel[n] *
    s_rel[n, k // group_size] (no requantisation)."""
    packed = _aligned(packed)
    Nn, Kp = packed.shape
    K = 2 * Kp
    dev = packed.device
    groups = s_rel.shape[1] if s_rel.dim() == 2 else -1
    if groups * group_size != K:
        raise ValueError(f"asym W4A8: {groups} scale groups of {group_size} do not cover K = {K}")
    codebook = codebook.to(device=dev, dtype=torch.float32).contiguous()
    s_channel = s_channel.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    s_rel = (s_rel if s_rel.dtype == torch.uint8 else s_rel.view(torch.uint8)).to(dev).contiguous()
    out = torch.empty((Nn, K), dtype=torch.float32, device=dev)
    if Nn and K:
        N.call("qlin_dequant_asym_w4a8", packed.data_ptr(), codebook.data_ptr(), s_channel.data_ptr(),
               s_rel.data_ptr(), int(group_size), Nn, K, out.data_ptr(), _stream(packed))
    return out


def _scale_arg(scale, n, device):
    s = scale.reshape(-1).to(device=device, dtype=torch.float32).contiguous() if torch.is_tensor(scale) \
        else torch.tensor([float(scale)], dtype=torch.float32, device=device)
    if s.numel() == 1:
        return s, N.WSCALE_TENSOR
    if s.numel() != n:
        raise ValueError(f"scale must have 1 or {n} entries, got {s.numel()}")
    return s, N.WSCALE_ROW


def dequant_int8(q: torch.Tensor, scale, rot=None) -> torch.Tensor:
    """float32 ``rotate_weight(q.float() * scale)`` (rotation optional)."""
    q = _aligned(q)
    Nn, K = q.shape
    out = torch.empty((Nn, K), dtype=torch.float32, device=q.device)
    if Nn and K:
        st = _stream(q)
        s, mode = _scale_arg(scale, Nn, q.device)
        kind, g, c = _rot_args(rot, torch.float32)
        N.call("qlin_dequant_int8", q.data_ptr(), s.data_ptr(), mode, Nn, K, kind, g, c, out.data_ptr(), st)
    return out


def requant_int8(w: torch.Tensor, scale, rot=None, stochastic=False, seed=0) -> torch.Tensor:
    """int8 ``quantize_int8(rotate_weight(w), scale)`` with the given (original)
    scale; stochastic=True follows stochastic_round_int8_delta's rule."""
    w = _aligned(w.to(torch.float32))
    Nn, K = w.shape
    q = torch.empty((Nn, K), dtype=torch.int8, device=w.device)
    if Nn and K:
        st = _stream(w)
        s, mode = _scale_arg(scale, Nn, w.device)
        kind, g, c = _rot_args(rot, torch.float32)
        N.call("qlin_requant_int8", w.data_ptr(), s.data_ptr(), mode, Nn, K, kind, g, c,
               N.ROUND_STOCHASTIC if stochastic else N.ROUND_NEAREST, int(seed) & (2 ** 64 - 1), q.data_ptr(), st)
    return q


def device_error(device=None) -> int:
    """Read and clear the device-side error word (bit 0: a GEMM pipeline
    wait timed out; bit 1: a row-kernel wait timed out; bit 2: a timed-out
    GEMM's in-flight work did not drain within the limit either)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    N.call("qlin_set_device", dev.index)
    bits = ctypes.c_uint32(0)
    N.call("qlin_device_error", torch.cuda.current_stream(dev).cuda_stream, ctypes.addressof(bits))
    return bits.value


def set_wait_limit(limit_ns: int = 0, device=None) -> None:
    """Wait limit of the kernels' bounded pipeline waits on ``device``, in
    nanoseconds (0: the default of 2 s)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    N.call("qlin_set_device", dev.index)
    N.call("qlin_set_wait_limit", int(limit_ns))


def selftest_wait_timeout(which: int) -> None:
    """Launch the one-thread bounded-wait self-test on the current stream:
    which 0 checks the GEMM pipeline wait, 1 the row kernels' wait."""
    N.call("qlin_selftest_wait_timeout", int(which), torch.cuda.current_stream().cuda_stream)


def selftest_gemm_stall(a_q, a_scale, w_q, w_scale, stall_kb: int = 0) -> torch.Tensor:
    """The W8A8 per-row GEMM (bf16 out, no bias) with K-slab ``stall_kb`` of
    each CTA's first tile never loaded: its wait runs out and the kernel
    returns with error bit 0 set.  Returns the (partly written) output."""
    _check_gemm(a_q, w_q)
    a_q, w_q = _aligned(a_q), _aligned(w_q)
    M, K = a_q.shape
    Nn = w_q.shape[0]
    out = torch.empty((M, Nn), dtype=torch.bfloat16, device=a_q.device)
    N.call("qlin_selftest_gemm_stall", _ptr(a_q), _ptr(a_scale.float().contiguous()), _ptr(w_q),
           _ptr(w_scale.float().contiguous()), _ptr(out), M, Nn, K, int(stall_kb), _stream(a_q))
    return out
