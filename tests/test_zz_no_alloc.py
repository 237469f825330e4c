"""The W8A8 GEMM entry point that allocates nothing (qlin_gemm_w8a8_splitk_noalloc).

Some callers cannot allocate device memory at the moment they run a GEMM:
an engine that reserves all of its GPU memory up front and forbids
allocations afterwards, or a plugin host that owns the allocator and hands
the kernel only its input and output buffers.  For them the split-K scratch
is a fixed array inside the library instead of a caller buffer.  These tests
call that entry point through the C ABI and check, on two calls in a row,
that its output is bit-identical to the ordinary qlin_gemm_w8a8 entry point
(the tolerance every W8A8 test here uses: none).  The array keeps the last
call's contents, so the second call also checks that a call starts from a
clean array.

The file name sorts last so a run that stops at the first failure has run
every other test before this one; it also passes on its own in a fresh
process.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]


def _inputs(seed, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    a_scale = torch.rand(M, device="cuda", generator=g) * 1e-3 + 1e-5
    w_scale = torch.rand(N, device="cuda", generator=g) * 1e-3 + 1e-5
    bias = (torch.randn(N, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
    return a, w, a_scale, w_scale, bias


def _call(native, name, a, w, a_scale, w_scale, bias, M, N, K):
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    native.call(name, a.data_ptr(), a_scale.data_ptr(), w.data_ptr(), w_scale.data_ptr(), native.WSCALE_ROW,
                bias.data_ptr(), out.data_ptr(), native.BF16, M, N, K, torch.cuda.current_stream().cuda_stream)
    return out


# (256, 1024, 16384) and (768, 1536, 24576) split K into three parts and use
# the fixed array; (1024, 3072, 3072) runs unsplit and needs none.
@pytest.mark.parametrize("M,N,K", [(256, 1024, 16384), (768, 1536, 24576), (1024, 3072, 3072)])
def test_no_alloc_entry_matches_the_allocating_entry(pkg, M, N, K):
    native = pkg._native
    scratch = ctypes.c_uint64(0)
    native.call("qlin_gemm_w8a8_splitk_scratch", M, N, K, ctypes.addressof(scratch))
    splits = scratch.value > 0
    assert splits == ((M, N, K) != (1024, 3072, 3072))
    a, w, a_scale, w_scale, bias = _inputs(7, M, N, K)
    want = _call(native, "qlin_gemm_w8a8", a, w, a_scale, w_scale, bias, M, N, K)
    for _ in range(2):
        got = _call(native, "qlin_gemm_w8a8_splitk_noalloc", a, w, a_scale, w_scale, bias, M, N, K)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.view(torch.int16).cpu().numpy(), want.view(torch.int16).cpu().numpy())
    assert pkg.ops.device_error() == 0
