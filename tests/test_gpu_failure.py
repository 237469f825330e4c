"""Failure detection on the GPU without a fault: bounded pipeline waits that
are made to run out return an error status the host reads, and the context
stays usable (a normal GEMM afterwards is still bit-exact).

The wait limit is lowered to a few milliseconds for these tests and restored
to its default afterwards.  Nothing here faults, traps or hangs a GPU: every
wait that runs out is a bounded loop that gives up after the limit.
"""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from conftest import cuda_ok
from oracle import qlinear_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


@pytest.fixture
def short_limit(pkg):
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    pkg.ops.set_wait_limit(5_000_000)  # 5 ms
    yield pkg
    pkg.ops.set_wait_limit(0)
    pkg.ops.device_error()


def _linear(P, M, N, K, seed):
    x = gi.activation(seed, M, K, "bf16")
    w = gi.weight(seed, N, K)
    wq, ws = O.quantize_int8_axiswise(w, 1)
    xq, xs = P.ops.quant_act_int8(torch.from_numpy(x).to(torch.bfloat16).cuda())
    return x, wq, ws, xq, xs


def _check_normal_gemm(P):
    x, wq, ws, xq, xs = _linear(P, 300, 520, 512, 41)
    y = P.ops.gemm_w8a8(xq, xs, torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(), None, torch.bfloat16)
    yo = O.int8_forward_dynamic_per_row(x, wq, ws, None, "bf16")
    np.testing.assert_array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), O.f32_to_bf16_bits(yo))
    assert P.ops.device_error() == 0


@pytest.mark.parametrize("which,bit", [(0, 1), (1, 2)])
def test_wait_selftest_times_out(short_limit, which, bit):
    P = short_limit
    P.ops.selftest_wait_timeout(which)
    torch.cuda.synchronize()
    assert P.ops.device_error() == bit
    _check_normal_gemm(P)


@pytest.mark.parametrize("M,N,K,stall_kb", [(512, 512, 1024, 3),  # CTA-pair kernel, all CTAs stall
                                            (128, 200, 512, 0)])  # single-CTA kernel
def test_gemm_stall_aborts_and_recovers(short_limit, M, N, K, stall_kb):
    P = short_limit
    _, wq, ws, xq, xs = _linear(P, M, N, K, 42)
    P.ops.selftest_gemm_stall(xq, xs, torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(), stall_kb)
    torch.cuda.synchronize()
    bits = P.ops.device_error()
    assert bits & 1, bits
    assert not bits & 4, bits  # the abort drained its in-flight loads and MMAs
    _check_normal_gemm(P)


def test_set_wait_limit_rejects_out_of_range(pkg):
    from comfyui_int8_fast_rocm_b200._native import NativeError
    with pytest.raises(NativeError):
        pkg.ops.set_wait_limit(10)  # below 1 us
    with pytest.raises(NativeError):
        pkg.ops.set_wait_limit(120 * 10**9)
