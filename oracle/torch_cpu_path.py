"""The reference's PyTorch CPU branch of the W8A8 ConvRot linear, restated
with the same torch calls -- TEST AND CPU-REFERENCE-ARM INFRASTRUCTURE ONLY.

This is what the reference runs when the activation is on the CPU
(int8_quant.py:148-164 with rotate_activation, convrot.py:89-118, and
quantize_int8_axiswise, int8_quant.py:41-52): a bf16 batched matmul for the
rotation, element-wise quantisation, ``torch._int_mm`` (oneDNN int8 on CPU)
and the two-rounding epilogue.  ``bench.py`` times it on the host cores as the
CPU baseline (``--impl reference`` and the ``cpu_baseline`` field); the tests
check that it agrees with the numpy oracle.  The product never imports it.
"""
from __future__ import annotations

import torch


def hadamard(size: int, kind: str) -> torch.Tensor:
    """Normalised Hadamard as built by convrot.build_hadamard (regular) or
    ``scipy.linalg.hadamard(size) / size**0.5`` (Sylvester), float32."""
    if kind == "regular":
        h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float32)
        h = h4
        while h.shape[0] < size:
            h = torch.kron(h, h4)
    else:
        h = torch.ones((1, 1), dtype=torch.float32)
        while h.shape[0] < size:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / (size ** 0.5)


def rotate_activation(x: torch.Tensor, H: torch.Tensor, group: int) -> torch.Tensor:
    """convrot.py:89-118."""
    shp = x.shape
    xg = x.view(*shp[:-1], shp[-1] // group, group)
    return torch.matmul(xg, H.to(dtype=x.dtype)).view(shp)


def quantize_int8_axiswise(x: torch.Tensor, dim: int):
    """int8_quant.py:41-52."""
    abs_max = x.abs().amax(dim=dim, keepdim=True)
    scale = (abs_max.float() / 127.0).clamp(min=1e-30)
    q = x.float().mul(1.0 / scale).round_().clamp_(-128.0, 127.0).to(torch.int8)
    return q, scale


@torch.no_grad()
def int8_forward_dynamic_per_row(x, weight, weight_scale, bias, compute_dtype):
    """int8_quant.py:148-164 (CPU branch)."""
    x_8, x_scale = quantize_int8_axiswise(x, dim=-1)
    res = torch._int_mm(x_8, weight.T)
    res_scaled = res.float().mul_(x_scale).mul_(weight_scale.T).to(compute_dtype)
    if bias is not None:
        res_scaled = res_scaled + bias.to(compute_dtype)
    return res_scaled


@torch.no_grad()
def convrot_w8a8_linear(x, H, group, weight, weight_scale, bias, compute_dtype):
    """Int8TensorwiseOps.Linear.forward's compute for a ConvRot layer
    (int8_quant.py:697-716) on CPU tensors."""
    x_2d = x.reshape(-1, x.shape[-1]).to(compute_dtype)
    if H is not None:
        x_2d = rotate_activation(x_2d, H, group)
    return int8_forward_dynamic_per_row(x_2d, weight, weight_scale, bias, compute_dtype)


# ---------------------------------------------------------------------------
# CPU baselines of the int4 configurations (timing only; bench.py
# --cpu-configs).  The row-wise W4A4 ConvRot linear is the reference's CPU
# restatement of convrot_w4a4_forward (int4_quant.py:292-353 with
# triton_int4_mm replaced by unpack + torch._int_mm, triton_int4_mm.py:4-9);
# the group-128 schemes have no reference and follow the oracle's
# restatement (group scales folded per 128-deep slab).
# ---------------------------------------------------------------------------


def _unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    """[N, K/2] int8 (low nibble = even k, signed) -> [N, K] int8."""
    p = packed.to(torch.int16) & 0xFF
    lo = ((p & 0xF) ^ 8) - 8
    hi = ((p >> 4) ^ 8) - 8
    return torch.stack((lo, hi), -1).reshape(packed.shape[0], -1).to(torch.int8)


def _pack_nibbles(q: torch.Tensor) -> torch.Tensor:
    u = q.to(torch.int16) & 0xF
    return (u[:, 0::2] | (u[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)


def _int4_groups(w: torch.Tensor, group: int = 128):
    """Symmetric int4 per row and 128-wide group: codes [N, K], scales [N, K/g]."""
    n, k = w.shape
    wg = w.reshape(n, k // group, group)
    s = (wg.abs().amax(-1).clamp(min=1e-10) / 7.0)
    q = (wg / s.unsqueeze(-1)).round().clamp(-7, 7).to(torch.int8).reshape(n, k)
    return q, s


def w4a8_g128_case(rows, n, k, gen):
    x = torch.randn((rows, k), generator=gen).to(torch.bfloat16)
    q, s = _int4_groups(torch.randn((n, k), generator=gen) * 0.02)
    packed, ws = _pack_nibbles(q), s.to(torch.bfloat16).float()
    bias = (torch.randn((n,), generator=gen) * 0.01).to(torch.bfloat16)

    def run():
        xq, xs = quantize_int8_axiswise(x, dim=-1)
        wq = _unpack_nibbles(packed)
        acc = torch.zeros((rows, n), dtype=torch.float32)
        for g in range(k // 128):
            part = torch._int_mm(xq[:, g * 128:(g + 1) * 128].contiguous(), wq[:, g * 128:(g + 1) * 128].T.contiguous())
            acc += part.float() * ws[:, g]
        return (acc * xs + bias.float()).to(torch.bfloat16)
    return run, n, k


def w4a4_g128_case(rows, n, k, gen):
    H = hadamard(128, "sylvester")
    x = torch.randn((rows, k), generator=gen).to(torch.bfloat16)
    q, s = _int4_groups(rotate_activation(torch.randn((n, k), generator=gen) * 0.02, H, 128))
    packed, ws = _pack_nibbles(q), s.to(torch.bfloat16).float()
    bias = (torch.randn((n,), generator=gen) * 0.01).to(torch.bfloat16)

    def run():
        xa, xsc = _int4_groups(rotate_activation(x, H, 128).float())
        wq = _unpack_nibbles(packed)
        acc = torch.zeros((rows, n), dtype=torch.float32)
        for g in range(k // 128):
            part = torch._int_mm(xa[:, g * 128:(g + 1) * 128].contiguous(), wq[:, g * 128:(g + 1) * 128].T.contiguous())
            acc += part.float() * (xsc[:, g:g + 1] * ws[:, g])
        return (acc + bias.float()).to(torch.bfloat16)
    return run, n, k


def w4a4_row_case(rows, n, k, gen):
    H = hadamard(256, "regular")
    x = torch.randn((rows, k), generator=gen).to(torch.bfloat16)
    wr = rotate_activation(torch.randn((n, k), generator=gen) * 0.02, H, 256)
    sw = wr.abs().amax(-1, keepdim=True).clamp(min=1e-10) / 7.0
    packed = _pack_nibbles((wr / sw).round().clamp(-7, 7).to(torch.int8))
    bias = (torch.randn((n,), generator=gen) * 0.01).to(torch.bfloat16)

    def run():
        xr = rotate_activation(x, H, 256)
        sa = xr.abs().amax(-1, keepdim=True).clamp(min=1e-10) / 7.0
        qa = (xr / sa).round().clamp(-7, 7).to(torch.int8)
        acc = torch._int_mm(qa, _unpack_nibbles(packed).T.contiguous())
        return (acc.float() * sa.float() * sw.reshape(1, -1) + bias.float()).to(torch.bfloat16)
    return run, n, k
