"""Seeded synthetic inputs shared by the golden generator and the tests.

Distributions follow the hot-path configurations: activations ~N(0,1) with
0.1% of the channels (at least one) scaled x20 as outliers, weights
~N(0, 0.02), biases ~N(0, 0.01).  Values are rounded to the compute dtype with
round-to-nearest-even so torch and numpy see bit-identical inputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle.qlinear_oracle import rnd  # noqa: E402


def activation(seed, M, K, dtype="bf16", zero_row=None, outlier_frac=0.001):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    n_out = max(1, int(round(K * outlier_frac)))
    cols = rng.permutation(K)[:n_out]
    x[:, cols] *= np.float32(20.0)
    if zero_row is not None:
        x[zero_row] = 0
    return rnd(dtype, x)


def weight(seed, N, K):
    rng = np.random.default_rng(1000 + seed)
    return (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)


def bias(seed, N, dtype="bf16"):
    rng = np.random.default_rng(2000 + seed)
    return rnd(dtype, rng.standard_normal(N, dtype=np.float32) * np.float32(0.01))


def int8_weight(seed, N, K):
    rng = np.random.default_rng(3000 + seed)
    return rng.integers(-127, 127, size=(N, K), dtype=np.int8)


def nibbles(seed, N, K):
    rng = np.random.default_rng(4000 + seed)
    return rng.integers(-8, 8, size=(N, K), dtype=np.int8)


def asym_w4a8(seed, N, K, group):
    """Packed unsigned codes [N,K/2] int8, codebook f32[16], s_channel f32[N],
    s_rel as float8_e4m3fn bytes [N, K/group] (positive normal values)."""
    rng = np.random.default_rng(5000 + seed)
    packed = rng.integers(0, 256, size=(N, K // 2), dtype=np.int64).astype(np.uint8).view(np.int8)
    codebook = np.sort(rng.standard_normal(16).astype(np.float32))
    s_ch = (np.abs(rng.standard_normal(N)) * 0.01 + 0.001).astype(np.float32)
    # e4m3 bytes with exponent field 5..9 (values 0.25..4), any mantissa
    e = rng.integers(5, 10, size=(N, K // group))
    m = rng.integers(0, 8, size=(N, K // group))
    s_rel = ((e << 3) | m).astype(np.uint8)
    return packed, codebook, s_ch, s_rel
