"""The kernels as ``torch.library`` custom operators (namespace ``qlin_b200``).

Every entry point of :mod:`ops` is registered as a custom op with a fake
(meta) implementation, so ``torch.compile`` traces a quantised linear as
opaque operator calls with known output shapes instead of breaking on the
ctypes call (``data_ptr()`` is not traceable).  The reference advertises
torch.compile support (README.md:19) and registers its own kitchen kernel
the same way (rocm_int8_kitchen_patch.py:19-21, ``torch.library.custom_op``).

The functions at the bottom keep the signatures of :mod:`ops` (a rotation is
``None`` or ``(kind, group)``) and call the registered operators; the
module surface (``int8_quant``, ``int4_quant``, ``kitchen_patch``, the
Triton-name shims, ``convrot``) goes through them.  The operators are
registered for CUDA only: a CPU tensor has no kernel and raises.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from . import ops

NS = "qlin_b200"


def _rot(kind: str, group: int):
    return None if kind == "none" else (kind, group)


def _rot_args(rot):
    if rot is None:
        return "none", 0
    kind, group = rot
    return str(kind), int(group)


def _rows_of(x: Tensor) -> int:
    if x.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(x.shape)}")
    return x.shape[0]


def _op(name, mutates_args=()):
    return torch.library.custom_op(f"{NS}::{name}", mutates_args=mutates_args, device_types="cuda")


# ---------------------------------------------------------------------------
# (a) activations
# ---------------------------------------------------------------------------


@_op("quant_act_int8")
def _quant_act_int8(x: Tensor, rot_kind: str, rot_group: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_act_int8(x, _rot(rot_kind, rot_group))


@_quant_act_int8.register_fake
def _(x, rot_kind, rot_group):
    M = _rows_of(x)
    return x.new_empty((M, x.shape[1]), dtype=torch.int8), x.new_empty((M, 1), dtype=torch.float32)


@_op("quant_act_int8_norm")
def _quant_act_int8_norm(x: Tensor, rot_kind: str, rot_group: int, norm: str, eps: float,
                         norm_weight: Optional[Tensor], mod_mul: Optional[Tensor], mod_add: Optional[Tensor],
                         rows_per_sample: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_act_int8_norm(x, _rot(rot_kind, rot_group), None if norm == "none" else norm, eps, norm_weight,
                                   mod_mul, mod_add, None if rows_per_sample < 0 else rows_per_sample)


@_quant_act_int8_norm.register_fake
def _(x, rot_kind, rot_group, norm, eps, norm_weight, mod_mul, mod_add, rows_per_sample):
    M = _rows_of(x)
    return x.new_empty((M, x.shape[1]), dtype=torch.int8), x.new_empty((M, 1), dtype=torch.float32)


@_op("quant_act_int8_cat")
def _quant_act_int8_cat(x1: Tensor, x2: Tensor, rot_kind: str, rot_group: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_act_int8_cat(x1, x2, _rot(rot_kind, rot_group))


@_quant_act_int8_cat.register_fake
def _(x1, x2, rot_kind, rot_group):
    M = _rows_of(x1)
    return (x1.new_empty((M, x1.shape[1] + x2.shape[1]), dtype=torch.int8),
            x1.new_empty((M, 1), dtype=torch.float32))


@_op("quant_act_int8_situ")
def _quant_act_int8_situ(x: Tensor, rot_kind: str, rot_group: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_act_int8_situ(x, _rot(rot_kind, rot_group))


@_quant_act_int8_situ.register_fake
def _(x, rot_kind, rot_group):
    M = _rows_of(x)
    return x.new_empty((M, x.shape[1] // 2), dtype=torch.int8), x.new_empty((M, 1), dtype=torch.float32)


@_op("qk_norm_rope_", mutates_args=("qkv",))
def _qk_norm_rope_(qkv: Tensor, heads: int, head_dim: int, q_weight: Optional[Tensor], k_weight: Optional[Tensor],
                   eps: float, cos: Optional[Tensor], sin: Optional[Tensor]) -> None:
    ops.qk_norm_rope_(qkv, heads, head_dim, q_weight, k_weight, eps, cos, sin)


@_qk_norm_rope_.register_fake
def _(qkv, heads, head_dim, q_weight, k_weight, eps, cos, sin):
    return None


@_op("quant_act_int4")
def _quant_act_int4(x: Tensor, rot_kind: str, rot_group: int, group: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_act_int4(x, _rot(rot_kind, rot_group), group)


@_quant_act_int4.register_fake
def _(x, rot_kind, rot_group, group):
    M = _rows_of(x)
    K = x.shape[1]
    return (x.new_empty((M, K), dtype=torch.int8),
            x.new_empty((M,) if group == 0 else (M, K // 128), dtype=torch.float32))


@_op("rotate")
def _rotate(x: Tensor, kind: str, group: int) -> Tensor:
    return ops.rotate(x, kind, group)


@_rotate.register_fake
def _(x, kind, group):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@_op("situ")
def _situ(x: Tensor) -> Tensor:
    return ops.situ(x)


@_situ.register_fake
def _(x):
    return x.new_empty((*x.shape[:-1], x.shape[-1] // 2))


# ---------------------------------------------------------------------------
# (b) / (c) GEMMs
# ---------------------------------------------------------------------------


@_op("gemm_w8a8")
def _gemm_w8a8(a_q: Tensor, a_scale: Tensor, w_q: Tensor, w_scale: Tensor, bias: Optional[Tensor],
               out_dtype: torch.dtype, per_row: bool) -> Tensor:
    return ops.gemm_w8a8(a_q, a_scale, w_q, w_scale, bias, out_dtype, per_row)


@_gemm_w8a8.register_fake
def _(a_q, a_scale, w_q, w_scale, bias, out_dtype, per_row):
    return a_q.new_empty((_rows_of(a_q), w_q.shape[0]), dtype=out_dtype)


@_op("gemm_w8a8_fused")
def _gemm_w8a8_fused(a_q: Tensor, a_scale: Tensor, w_q: Tensor, w_scale: Tensor, bias: Optional[Tensor],
                     out_dtype: torch.dtype, per_row: bool, gelu_from: int, residual: Optional[Tensor],
                     gate: Optional[Tensor], rows_per_gate: int) -> Tensor:
    return ops.gemm_w8a8_fused(a_q, a_scale, w_q, w_scale, bias, out_dtype, per_row,
                               None if gelu_from < 0 else gelu_from, residual, gate,
                               None if rows_per_gate < 0 else rows_per_gate)


@_gemm_w8a8_fused.register_fake
def _(a_q, a_scale, w_q, w_scale, bias, out_dtype, per_row, gelu_from, residual, gate, rows_per_gate):
    return a_q.new_empty((_rows_of(a_q), w_q.shape[0]), dtype=out_dtype)


@_op("gemm_w8a8_fused_into", mutates_args=("out",))
def _gemm_w8a8_fused_into(a_q: Tensor, a_scale: Tensor, w_q: Tensor, w_scale: Tensor, bias: Optional[Tensor],
                          out: Tensor, per_row: bool, gelu_from: int, residual: Optional[Tensor],
                          gate: Optional[Tensor], rows_per_gate: int, seg_rows: int, seg_stride: int,
                          seg_off: int) -> None:
    ops.gemm_w8a8_fused(a_q, a_scale, w_q, w_scale, bias, out.dtype, per_row,
                        None if gelu_from < 0 else gelu_from, residual, gate,
                        None if rows_per_gate < 0 else rows_per_gate, out=out,
                        out_rows=None if seg_rows <= 0 else (seg_rows, seg_stride, seg_off))


@_op("int_mm")
def _int_mm(a_q: Tensor, w_q: Tensor) -> Tensor:
    return ops.int_mm(a_q, w_q)


@_int_mm.register_fake
def _(a_q, w_q):
    return a_q.new_empty((_rows_of(a_q), w_q.shape[0]), dtype=torch.int32)


@_op("int4_mm")
def _int4_mm(a_q: Tensor, w_packed: Tensor) -> Tensor:
    return ops.int4_mm(a_q, w_packed)


@_int4_mm.register_fake
def _(a_q, w_packed):
    return a_q.new_empty((_rows_of(a_q), w_packed.shape[0]), dtype=torch.int32)


@_op("gemm_w4a4")
def _gemm_w4a4(a_q: Tensor, a_scale: Tensor, w_packed: Tensor, w_scale: Tensor, bias: Optional[Tensor],
               out_dtype: torch.dtype) -> Tensor:
    return ops.gemm_w4a4(a_q, a_scale, w_packed, w_scale, bias, out_dtype)


@_gemm_w4a4.register_fake
def _(a_q, a_scale, w_packed, w_scale, bias, out_dtype):
    return a_q.new_empty((_rows_of(a_q), w_packed.shape[0]), dtype=out_dtype)


@_op("gemm_w4_g128")
def _gemm_w4_g128(a_q: Tensor, a_scale: Tensor, w_packed: Tensor, w_gscale: Tensor, bias: Optional[Tensor],
                  out_dtype: torch.dtype, a_int4_groups: bool) -> Tensor:
    return ops.gemm_w4_g128(a_q, a_scale, w_packed, w_gscale, bias, out_dtype, a_int4_groups)


@_gemm_w4_g128.register_fake
def _(a_q, a_scale, w_packed, w_gscale, bias, out_dtype, a_int4_groups):
    return a_q.new_empty((_rows_of(a_q), w_packed.shape[0]), dtype=out_dtype)


# ---------------------------------------------------------------------------
# (d) weights
# ---------------------------------------------------------------------------


@_op("quant_weight_int8")
def _quant_weight_int8(w: Tensor, rot_kind: str, rot_group: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_weight_int8(w, _rot(rot_kind, rot_group))


@_quant_weight_int8.register_fake
def _(w, rot_kind, rot_group):
    Nn = _rows_of(w)
    return w.new_empty((Nn, w.shape[1]), dtype=torch.int8), w.new_empty((Nn, 1), dtype=torch.float32)


@_op("quant_weight_int4")
def _quant_weight_int4(w: Tensor, rot_kind: str, rot_group: int, group: int) -> Tuple[Tensor, Tensor]:
    return ops.quant_weight_int4(w, _rot(rot_kind, rot_group), group)


@_quant_weight_int4.register_fake
def _(w, rot_kind, rot_group, group):
    Nn = _rows_of(w)
    K = w.shape[1]
    return (w.new_empty((Nn, K // 2), dtype=torch.int8),
            w.new_empty((Nn,) if group == 0 else (Nn, K // 128), dtype=torch.float32))


@_op("requant_asym_w4a8")
def _requant_asym_w4a8(packed: Tensor, codebook: Tensor, s_channel: Tensor, s_rel: Tensor,
                       group_size: int) -> Tuple[Tensor, Tensor]:
    return ops.requant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size)


@_requant_asym_w4a8.register_fake
def _(packed, codebook, s_channel, s_rel, group_size):
    Nn = _rows_of(packed)
    return (packed.new_empty((Nn, 2 * packed.shape[1]), dtype=torch.int8),
            packed.new_empty((Nn, 1), dtype=torch.float32))


@_op("dequant_asym_w4a8")
def _dequant_asym_w4a8(packed: Tensor, codebook: Tensor, s_channel: Tensor, s_rel: Tensor,
                       group_size: int) -> Tensor:
    return ops.dequant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size)


@_dequant_asym_w4a8.register_fake
def _(packed, codebook, s_channel, s_rel, group_size):
    return packed.new_empty((_rows_of(packed), 2 * packed.shape[1]), dtype=torch.float32)


@_op("dequant_int8")
def _dequant_int8(q: Tensor, scale: Tensor, rot_kind: str, rot_group: int) -> Tensor:
    return ops.dequant_int8(q, scale, _rot(rot_kind, rot_group))


@_dequant_int8.register_fake
def _(q, scale, rot_kind, rot_group):
    return q.new_empty((_rows_of(q), q.shape[1]), dtype=torch.float32)


@_op("requant_int8")
def _requant_int8(w: Tensor, scale: Tensor, rot_kind: str, rot_group: int, stochastic: bool, seed: int) -> Tensor:
    return ops.requant_int8(w, scale, _rot(rot_kind, rot_group), stochastic, seed & (2 ** 64 - 1))


@_requant_int8.register_fake
def _(w, scale, rot_kind, rot_group, stochastic, seed):
    return w.new_empty((_rows_of(w), w.shape[1]), dtype=torch.int8)


# ---------------------------------------------------------------------------
# callers' view: the signatures of ops.*, through the registered operators
# ---------------------------------------------------------------------------

_L = getattr(torch.ops, NS)


def _scale_tensor(scale, device):
    return scale if torch.is_tensor(scale) else torch.tensor([float(scale)], dtype=torch.float32, device=device)


def _signed64(v: int) -> int:
    v = int(v) & (2 ** 64 - 1)
    return v - 2 ** 64 if v >= 2 ** 63 else v


def quant_act_int8(x: Tensor, rot=None):
    return _L.quant_act_int8(x, *_rot_args(rot))


def quant_act_int8_norm(x: Tensor, rot=None, norm=None, eps: float = 1e-6, norm_weight=None, mod_mul=None,
                        mod_add=None, rows_per_sample=None):
    return _L.quant_act_int8_norm(x, *_rot_args(rot), "none" if norm is None else str(norm), float(eps),
                                  norm_weight, mod_mul, mod_add, -1 if rows_per_sample is None else int(rows_per_sample))


def quant_act_int8_cat(x1: Tensor, x2: Tensor, rot=None):
    return _L.quant_act_int8_cat(x1, x2, *_rot_args(rot))


def quant_act_int8_situ(x: Tensor, rot=None):
    return _L.quant_act_int8_situ(x, *_rot_args(rot))


def qk_norm_rope_(qkv: Tensor, heads: int, head_dim: int, q_weight=None, k_weight=None, eps: float = 1e-6,
                  cos=None, sin=None) -> Tensor:
    _L.qk_norm_rope_(qkv, int(heads), int(head_dim), q_weight, k_weight, float(eps), cos, sin)
    return qkv


def quant_act_int4(x: Tensor, rot=None, group: int = 0):
    return _L.quant_act_int4(x, *_rot_args(rot), int(group))


def rotate(x: Tensor, kind: str, group: int) -> Tensor:
    return _L.rotate(x, str(kind), int(group))


def situ(x: Tensor) -> Tensor:
    return _L.situ(x)


def gemm_w8a8(a_q, a_scale, w_q, w_scale, bias=None, out_dtype=torch.bfloat16, per_row=True):
    return _L.gemm_w8a8(a_q, a_scale, w_q, w_scale, bias, out_dtype, bool(per_row))


def gemm_w8a8_fused(a_q, a_scale, w_q, w_scale, bias=None, out_dtype=torch.bfloat16, per_row=True, gelu_from=None,
                    residual=None, gate=None, rows_per_gate=None, out=None, out_rows=None):
    if out is None:
        if out_rows is not None:
            raise ValueError("out_rows needs out")
        return _L.gemm_w8a8_fused(a_q, a_scale, w_q, w_scale, bias, out_dtype, bool(per_row),
                                  -1 if gelu_from is None else int(gelu_from), residual, gate,
                                  -1 if rows_per_gate is None else int(rows_per_gate))
    if out.dtype != out_dtype:
        raise ValueError(f"out is {out.dtype}, the GEMM writes {out_dtype}")
    n, stride, off = (0, 0, 0) if out_rows is None else (int(v) for v in out_rows)
    _L.gemm_w8a8_fused_into(a_q, a_scale, w_q, w_scale, bias, out, bool(per_row),
                            -1 if gelu_from is None else int(gelu_from), residual, gate,
                            -1 if rows_per_gate is None else int(rows_per_gate), n, stride, off)
    return out


def int_mm(a_q, w_q):
    return _L.int_mm(a_q, w_q)


def int4_mm(a_q, w_packed):
    return _L.int4_mm(a_q, w_packed)


def gemm_w4a4(a_q, a_scale, w_packed, w_scale, bias=None, out_dtype=torch.bfloat16):
    return _L.gemm_w4a4(a_q, a_scale, w_packed, w_scale, bias, out_dtype)


def gemm_w4_g128(a_q, a_scale, w_packed, w_gscale, bias=None, out_dtype=torch.bfloat16, a_int4_groups=False):
    return _L.gemm_w4_g128(a_q, a_scale, w_packed, w_gscale, bias, out_dtype, bool(a_int4_groups))


def quant_weight_int8(w: Tensor, rot=None):
    return _L.quant_weight_int8(w, *_rot_args(rot))


def quant_weight_int4(w: Tensor, rot=None, group: int = 0):
    return _L.quant_weight_int4(w, *_rot_args(rot), int(group))


def requant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size: int):
    return _L.requant_asym_w4a8(packed, codebook, s_channel, s_rel, int(group_size))


def dequant_asym_w4a8(packed, codebook, s_channel, s_rel, group_size: int) -> Tensor:
    return _L.dequant_asym_w4a8(packed, codebook, s_channel, s_rel, int(group_size))


def dequant_int8(q: Tensor, scale, rot=None) -> Tensor:
    return _L.dequant_int8(q, _scale_tensor(scale, q.device), *_rot_args(rot))


def requant_int8(w: Tensor, scale, rot=None, stochastic=False, seed=0) -> Tensor:
    return _L.requant_int8(w, _scale_tensor(scale, w.device), *_rot_args(rot), bool(stochastic), _signed64(seed))


hadamard_scale = ops.hadamard_scale
device_error = ops.device_error
