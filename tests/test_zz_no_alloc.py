"""fw_linear_e4m3_noalloc: the e4m3 linear layer for callers that cannot allocate device memory.

Such callers (a host whose GPU memory is entirely owned by another framework's pool, or a
latency-critical loop that must not call cudaMalloc) get the quantised activations kept in a
fixed array inside the library instead of caller-provided scratch.  This file runs last so that
a failure here never hides another test; it must pass alone in a fresh process and after the
rest.  The result is compared, through the C ABI, with the allocating path (fw_quant_e4m3 into
torch-allocated scratch, then fw_gemm_e4m3) on two different problems called back to back, so a
stale scratch from the first call would show up in the second.  Same kernels, same inputs:
the outputs must be identical (tolerance 0).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    bias = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    return x, w, bias


def test_noalloc_matches_allocating_path():
    from fastworld_b200 import ops
    from fastworld_b200._lib import check, lib, ptr, stream_ptr
    for M, N, K, seed in ((2640, 1536, 1536, 0), (700, 1024, 8960, 1)):
        x, w, bias = _problem(M, N, K, seed)
        w8, sw = ops.quant_e4m3(w)
        a8, sa = ops.quant_e4m3(x)                       # allocating path: caller scratch
        ref = ops.gemm_e4m3(a8, sa, w8, sw, bias)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        check(lib().fw_linear_e4m3_noalloc(ptr(x), ptr(w8), ptr(sw), ptr(bias), ptr(out), M, N, K, stream_ptr()),
              "fw_linear_e4m3_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_noalloc_rejects_oversized_problems():
    from fastworld_b200._lib import lib
    x = torch.zeros(16, 16, device="cuda", dtype=torch.bfloat16)
    # 4096 x 9216 bytes > 32 MiB: rejected on the host before any launch
    assert lib().fw_linear_e4m3_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, x.data_ptr(), 4096, 64, 9216,
                                        None) == -9
    assert lib().fw_linear_e4m3_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, x.data_ptr(), 20000, 64, 16,
                                        None) == -9
