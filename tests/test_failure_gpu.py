"""Failure detection on one GPU without a fault: bounded device waits that nothing satisfies
run out, record their code in the status word, unwind, and the context keeps working.

The engine's kernels bound every wait (an mbarrier in the tcgen05 GEMM and attention kernels,
another rank's epoch flag in the tensor-parallel reductions); on timeout they record a status
code that the host reads after synchronising.  ``fw_selftest_wait`` drives both kinds with a
short limit: an mbarrier that no thread or copy completes, in CTAs that hold Tensor Memory, and
the real two-rank reduction kernel run as rank 0 of a group whose other rank never runs.  After
each, a tcgen05 GEMM (which allocates Tensor Memory again) must still match torch."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_TEST, DEV_TIMEOUT_PEER = 6, 7
LIMIT_NS = 10_000_000   # 10 ms


def run_selftest(which):
    from fastworld_b200._lib import check, lib, stream_ptr
    L = lib()
    nb = L.fw_selftest_bytes(which)
    scratch = torch.zeros((nb + 255) // 256 * 256, dtype=torch.uint8, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    check(L.fw_selftest_wait(which, LIMIT_NS, ctypes.c_void_p(scratch.data_ptr()), scratch.numel(),
                             ctypes.c_void_p(status.data_ptr()), stream_ptr()), "fw_selftest_wait")
    e1.record()
    torch.cuda.synchronize()
    return status.cpu(), scratch, e0.elapsed_time(e1)


def gemm_still_correct():
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.randn(300, 256, device="cuda", generator=g).bfloat16()
    B = torch.randn(512, 256, device="cuda", generator=g).bfloat16()
    out = ops.gemm(A, B, None, "none")
    ref = A.float() @ B.float().t()
    torch.cuda.synchronize()
    return float((out.float() - ref).norm() / ref.norm())


def test_mbarrier_wait_runs_out_and_unwinds():
    status, scratch, ms = run_selftest(0)
    assert int(status[0]) == DEV_TIMEOUT_TEST
    outcome = scratch[:4 * 2 * 4].view(torch.int32).cpu()
    assert outcome.tolist() == [2] * 8          # every waiter of every CTA gave up (none returned "ok")
    assert LIMIT_NS / 1e6 <= ms < 1000.0        # ran out after the limit, long before the 2 s default
    assert gemm_still_correct() < 6e-3          # Tensor Memory was freed; the context works


def test_peer_flag_wait_runs_out_and_kernel_completes():
    status, _, ms = run_selftest(1)
    assert int(status[0]) == DEV_TIMEOUT_PEER
    assert 2 * LIMIT_NS / 1e6 <= ms < 1000.0    # both phases waited out their limit, then returned
    assert gemm_still_correct() < 6e-3


def test_limits_are_validated():
    from fastworld_b200._lib import lib
    L = lib()
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert L.fw_selftest_wait(0, 0, ctypes.c_void_p(buf.data_ptr()), 4096, ctypes.c_void_p(st.data_ptr()),
                              None) == -1
    assert L.fw_selftest_wait(1, LIMIT_NS, ctypes.c_void_p(buf.data_ptr()), 16, ctypes.c_void_p(st.data_ptr()),
                              None) == -8
