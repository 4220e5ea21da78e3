"""Small, self-terminating workloads for ncu captures (run them plain first, then under ncu).

    python -m fastworld_b200.profile chunk [--chunks 2] [--config mg2|mg2_fp8]   eager chunks (chunk 0, then steady)
    python -m fastworld_b200.profile gemm  [--reps 3]     FFN-up GEMM, MG2 shape, GELU epilogue
    python -m fastworld_b200.profile gemm_resid           O-projection GEMM (N = K = 1536) with the gated residual
    python -m fastworld_b200.profile attn  [--reps 3]     steady self-attention, 12 heads, 2640 + 2640 keys
    python -m fastworld_b200.profile fp8_peak             dense e4m3 peak: a library GEMM (cuBLASLt via
                                                          torch._scaled_mm) at 8192^3, best of 10, next to
                                                          this library's e4m3 GEMM at the same size
"""
from __future__ import annotations

import argparse

import torch


def chunk(n: int, config: str = "mg2") -> None:
    from fastworld_b200 import _lib
    from fastworld_b200.config import PRESETS
    from fastworld_b200.static import B200StaticMG
    S = B200StaticMG(PRESETS[config], seed=0)
    S.add_image("img0", seed=3, max_chunks=n + 1)
    path = [("img0", ("w", "u"))] * (n + 1)
    for k in range(n):
        S._prep(path, k)
        c0 = _lib.lib().fw_launch_count()
        S._chunk(k == 0)
        torch.cuda.synchronize()
        print(f"chunk {k}: {_lib.lib().fw_launch_count() - c0} launches, status {S.device_status()}")


def gemm(reps: int) -> None:
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(2640, 1536, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(8960, 1536, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(8960, device="cuda", dtype=torch.bfloat16)
    for _ in range(reps):
        ops.gemm(A, B, bias, "gelu_tanh")
    torch.cuda.synchronize()
    print("gemm ok")


def gemm_resid(reps: int) -> None:
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(2640, 1536, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(1536, 1536, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(1536, device="cuda", dtype=torch.bfloat16)
    resid = torch.zeros(2640, 1536, device="cuda")
    gate = torch.ones(3, 1536, device="cuda")
    for _ in range(reps):
        ops.gemm_resid_(resid, A, B, bias, gate, 880)
    torch.cuda.synchronize()
    print("gemm_resid ok")


def attn(reps: int) -> None:
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    r = lambda n: torch.randn(n, 12, 128, device="cuda", generator=g).to(torch.bfloat16)
    q, k0, v0, k1, v1 = r(2640), r(2640), r(2640), r(2640), r(2640)
    meta = torch.tensor([2640, 2640], dtype=torch.int32, device="cuda")
    for _ in range(reps):
        ops.attention(q, k0, v0, k1, v1, meta)
    torch.cuda.synchronize()
    print("attn ok")


def fp8_peak(reps: int) -> None:
    from fastworld_b200 import ops
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(n, n, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(n, n, device="cuda", generator=g).to(torch.bfloat16)
    a8, sa = ops.quant_e4m3(a)
    b8, sw = ops.quant_e4m3(b)
    fa, fb = a8.view(torch.float8_e4m3fn), b8.view(torch.float8_e4m3fn)
    one = torch.ones((), device="cuda")

    def best(fn, n_rep=10):
        for _ in range(3):
            fn()
        t = 1e9
        for _ in range(n_rep):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            t = min(t, e0.elapsed_time(e1))
        return t
    flop = 2.0 * n ** 3
    t_lib = best(lambda: torch._scaled_mm(fa, fb.t(), one, one, out_dtype=torch.bfloat16))
    t_ours = best(lambda: ops.gemm_e4m3(a8, sa, b8, sw, None, "none"))
    t_bf16 = best(lambda: torch.matmul(a, b.t()))
    print(f"e4m3 8192^3: library {flop / t_lib / 1e9:.1f} TFLOP/s, fastworld_b200 {flop / t_ours / 1e9:.1f} TFLOP/s; "
          f"bf16 library {flop / t_bf16 / 1e9:.1f} TFLOP/s (burst, best of 10)")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["chunk", "gemm", "gemm_resid", "attn", "fp8_peak"])
    ap.add_argument("--chunks", type=int, default=2)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--config", default="mg2")
    a = ap.parse_args()
    {"chunk": lambda: chunk(a.chunks, a.config), "gemm": lambda: gemm(a.reps), "gemm_resid": lambda: gemm_resid(a.reps),
     "attn": lambda: attn(a.reps), "fp8_peak": lambda: fp8_peak(a.reps)}[a.what]()
