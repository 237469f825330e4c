"""The oracle's restatement of the eager neighbours of a DiT linear (row
norms, modulation, GELU, gated residual) against torch's own CPU kernels on
the same bf16 / f16 tensors.  No GPU needed."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import qlinear_oracle as O

TDT = {"bf16": torch.bfloat16, "f16": torch.float16}


def _x(rng, shape, dt, scale=1.0, offset=0.0):
    return O.rnd(dt, rng.standard_normal(shape).astype(np.float32) * scale + offset)


def _t(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a)).to(TDT[dt])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_layer_norm_modulation_matches_torch(dt):
    """``layer_norm(x) * (1 + scale) + shift`` per sample: the oracle's
    float64-summed statistics differ from torch's float32 ones only in rare
    last-unit roundings (<= 0.01% of values, 1 unit)."""
    rng = np.random.default_rng(0)
    S, L, K = 2, 96, 3072
    x = _x(rng, (S * L, K), dt, 2.0, 0.3)
    scale, shift = _x(rng, (S, K), dt, 0.3), _x(rng, (S, K), dt, 0.2)
    xt = _t(x, dt).view(S, L, K)
    mul = 1 + _t(scale, dt)
    ref = (F.layer_norm(xt, (K,), eps=1e-6) * mul[:, None] + _t(shift, dt)[:, None]).reshape(S * L, K)
    got = O.norm_modulate(x, dt, norm="layer", eps=1e-6, mod_mul=mul.float().numpy(), mod_add=shift,
                          rows_per_sample=L)
    diff = ref.float().numpy() != got
    assert diff.mean() <= 1e-4, diff.mean()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("with_weight", [True, False])
def test_rms_norm_matches_torch(dt, with_weight):
    rng = np.random.default_rng(1)
    x = _x(rng, (128, 2048), dt, 1.5)
    w = _x(rng, 2048, dt, 0.5, 1.0) if with_weight else None
    ref = F.rms_norm(_t(x, dt), (2048,), None if w is None else _t(w, dt), 1e-6).float().numpy()
    got = O.row_norm(x, "rms", 1e-6, dt, w)
    assert (ref != got).mean() <= 1e-4


def gelu_close(got, ref, dt):
    """One unit of ``dt`` relative, or 2^-20 absolute (where tanh saturates,
    one library returns -0.0 and another a value of order -1e-7)."""
    unit = 2.0 ** -7 if dt == "bf16" else 2.0 ** -10
    return np.abs(got - ref) <= np.maximum(np.abs(ref) * unit, 2.0 ** -20)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_gelu_tanh_matches_torch(dt):
    """The oracle's GELU is the exact tanh-form function: equal to torch's
    float64 ``F.gelu(approximate="tanh")`` rounded to float32 and to the
    dtype wherever |value| > 2^-30 (<= 0.01% last-unit differences from the
    two float64 evaluation orders; below that torch's float64 tanh form
    cancels to 0 for x < -7); torch's own 16-bit CPU kernel is within
    ``gelu_close`` of it."""
    rng = np.random.default_rng(2)
    x = _x(rng, (256, 1024), dt, 3.0)
    exact = F.gelu(torch.from_numpy(x).double(), approximate="tanh").float().numpy()
    got = O.gelu_tanh(x)
    big = np.abs(got) > 2.0 ** -30
    assert (O.rnd(dt, exact)[big] != O.rnd(dt, got)[big]).mean() <= 1e-4
    assert (np.abs(exact[~big]) <= 2.0 ** -30).all()
    ref16 = F.gelu(_t(x, dt), approximate="tanh").float().numpy()
    assert gelu_close(O.rnd(dt, got), ref16, dt).all()


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_gated_residual_matches_torch(dt):
    rng = np.random.default_rng(3)
    S, L, N = 3, 40, 512
    y, res = _x(rng, (S * L, N), dt), _x(rng, (S * L, N), dt, 2.0)
    gate = _x(rng, (S, N), dt, 0.5)
    ref = (_t(res, dt).view(S, L, N) + _t(gate, dt)[:, None] * _t(y, dt).view(S, L, N)).reshape(S * L, N)
    got = O.linear_post(y, dt, residual=res, gate=gate, rows_per_gate=L)
    np.testing.assert_array_equal(ref.float().numpy(), got)
    np.testing.assert_array_equal((_t(res, dt) + _t(y, dt)).float().numpy(), O.linear_post(y, dt, residual=res))


def _rope_tables(L, hd):
    inv = 1.0 / (10000.0 ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    ang = np.arange(L, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_qk_norm_rope_matches_torch(dt):
    """q/k RMSNorm + float32 rotary embedding (Flux's apply_rope) in torch's
    CPU kernels vs the oracle: rare last-unit differences from the norm's
    float32 statistics only."""
    rng = np.random.default_rng(4)
    B, L, H, hd = 2, 48, 3, 128
    qkv = _x(rng, (B * L, 3 * H * hd + 32), dt, 1.5)
    qw, kw = _x(rng, hd, dt, 0.3, 1.0), _x(rng, hd, dt, 0.3, 1.0)
    cos, sin = _rope_tables(L, hd)
    t = _t(qkv, dt).view(B, L, -1)
    q, k, v = t[..., :3 * H * hd].reshape(B, L, 3, H, hd).permute(2, 0, 3, 1, 4)

    def rope(x):
        a, b = x[..., 0::2].float(), x[..., 1::2].float()
        c, s = torch.from_numpy(cos), torch.from_numpy(sin)
        return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2).to(x.dtype)

    rq = rope(F.rms_norm(q, (hd,), _t(qw, dt), 1e-6)).transpose(1, 2).reshape(B * L, H * hd)
    rk = rope(F.rms_norm(k, (hd,), _t(kw, dt), 1e-6)).transpose(1, 2).reshape(B * L, H * hd)
    got = O.qk_norm_rope(qkv, H, hd, dt, qw, kw, 1e-6, cos, sin, positions=L)
    assert (rq.float().numpy() != got[:, :H * hd]).mean() <= 1e-3
    assert (rk.float().numpy() != got[:, H * hd:2 * H * hd]).mean() <= 1e-3
    np.testing.assert_array_equal(got[:, 2 * H * hd:], qkv[:, 2 * H * hd:])
