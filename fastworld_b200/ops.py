"""Torch-facing wrappers of the op-level C ABI (device tensors in, device tensors out).

These call the sm_100a kernels directly; there is no fallback: a tensor on the wrong device
or with the wrong dtype/layout raises.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_ptr

EPILOGUES = {"none": _lib.EPI_BF16, "gelu_tanh": _lib.EPI_GELU_BF16, "f32": _lib.EPI_F32,
             "gelu_erf": _lib.EPI_GELU_ERF_BF16}


def _req(t, dtype, name):
    if not (t.is_cuda and t.dtype == dtype and t.is_contiguous()):
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor, got {t.dtype} on {t.device}")


def gemm(a: torch.Tensor, b: torch.Tensor, bias=None, epilogue: str = "none", tile_n: int = 0) -> torch.Tensor:
    """a [M, K] @ b[N, K]^T (+ bias) with fp32 accumulation; bf16 (or fp32 for 'f32') output."""
    _req(a, torch.bfloat16, "a")
    _req(b, torch.bfloat16, "b")
    if bias is not None:
        _req(bias, torch.bfloat16, "bias")
    M, K = a.shape
    N = b.shape[0]
    out = torch.empty(M, N, device=a.device, dtype=torch.float32 if epilogue == "f32" else torch.bfloat16)
    check(lib().fw_gemm_bf16(ptr(a), ptr(b), ptr(bias), ptr(out), M, N, K, EPILOGUES[epilogue], tile_n,
                             stream_ptr()), "gemm")
    return out


def quant_e4m3(x: torch.Tensor):
    """Per-row e4m3 quantisation: returns (q [M, K] uint8 e4m3 bits, scale [M] fp32)."""
    _req(x, torch.bfloat16, "x")
    M, K = x.shape
    q = torch.empty(M, K, device=x.device, dtype=torch.uint8)
    sc = torch.empty(M, device=x.device, dtype=torch.float32)
    check(lib().fw_quant_e4m3(ptr(x), M, K, ptr(q), ptr(sc), stream_ptr()), "quant_e4m3")
    return q, sc


def gemm_e4m3(a8: torch.Tensor, sa: torch.Tensor, b8: torch.Tensor, sw: torch.Tensor, bias=None,
              epilogue: str = "none", tile_n: int = 0) -> torch.Tensor:
    """(a8 [M, K] e4m3 * sa[M]) @ (b8 [N, K] e4m3 * sw[N])^T (+ bias), fp32 accumulation."""
    for n, t, d in (("a8", a8, torch.uint8), ("b8", b8, torch.uint8), ("sa", sa, torch.float32),
                    ("sw", sw, torch.float32)):
        _req(t, d, n)
    M, K = a8.shape
    N = b8.shape[0]
    out = torch.empty(M, N, device=a8.device, dtype=torch.float32 if epilogue == "f32" else torch.bfloat16)
    check(lib().fw_gemm_e4m3(ptr(a8), ptr(sa), ptr(b8), ptr(sw), ptr(bias), ptr(out), M, N, K, EPILOGUES[epilogue],
                             tile_n, stream_ptr()), "gemm_e4m3")
    return out


def gemm_resid_(resid: torch.Tensor, a: torch.Tensor, b: torch.Tensor, bias=None, gate=None,
                rows_per_frame: int = 1 << 30) -> torch.Tensor:
    """resid (fp32, in place) += gate[row // rows_per_frame] * (a @ b^T + bias)."""
    _req(resid, torch.float32, "resid")
    _req(a, torch.bfloat16, "a")
    _req(b, torch.bfloat16, "b")
    if gate is not None:
        _req(gate, torch.float32, "gate")
    M, K = a.shape
    N = b.shape[0]
    check(lib().fw_gemm_bf16_resid(ptr(a), ptr(b), ptr(bias), ptr(resid), ptr(gate), rows_per_frame, M, N, K,
                                   stream_ptr()), "gemm_resid")
    return resid


def attention(q: torch.Tensor, k0: torch.Tensor, v0: torch.Tensor, k1: torch.Tensor, v1: torch.Tensor,
              meta: torch.Tensor, status: torch.Tensor = None) -> torch.Tensor:
    """Non-causal attention of q [Lq, H, 128] over keys [k0[:n0] | k1[:n1]] with
    meta = device int32 (n0, n1).  Returns [Lq, H * 128] bf16."""
    for n, t in (("q", q), ("k0", k0), ("v0", v0), ("k1", k1), ("v1", v1)):
        _req(t, torch.bfloat16, n)
    _req(meta, torch.int32, "meta")
    Lq, H, Dh = q.shape
    assert Dh == 128
    out = torch.empty(Lq, H * Dh, device=q.device, dtype=torch.bfloat16)
    check(lib().fw_attention(ptr(q), Lq, H, ptr(k0), ptr(v0), k0.shape[0], ptr(k1), ptr(v1), k1.shape[0], ptr(meta),
                             ptr(out), ptr(status), stream_ptr()), "attention")
    return out


def copy_(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """Byte copy src -> dst with the vectorised copy kernel (same byte size)."""
    nb = dst.numel() * dst.element_size()
    if src.numel() * src.element_size() != nb or not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("copy_: contiguous tensors of equal byte size required")
    check(lib().fw_copy(ptr(dst), ptr(src), nb, stream_ptr()), "copy")
    return dst


def layernorm(x: torch.Tensor, eps: float = 1e-6, shift=None, scale=None, w=None, b=None, out=None) -> torch.Tensor:
    """bf16 LN(x) of fp32 rows x [M, D], then * (1 + scale) + shift (fp32 [D]) or * w + b (bf16 [D])."""
    _req(x, torch.float32, "x")
    for n, t, d in (("shift", shift, torch.float32), ("scale", scale, torch.float32), ("w", w, torch.bfloat16),
                    ("b", b, torch.bfloat16)):
        if t is not None:
            _req(t, d, n)
    M, D = x.shape
    out = torch.empty(M, D, device=x.device, dtype=torch.bfloat16) if out is None else out
    _req(out, torch.bfloat16, "out")
    check(lib().fw_layernorm(ptr(x), M, D, float(eps), ptr(shift), ptr(scale), ptr(w), ptr(b), ptr(out),
                             stream_ptr()), "layernorm")
    return out


def rms_rope(x: torch.Tensor, w: torch.Tensor, rope=None, head_dim: int = 128, eps: float = 1e-6,
             out=None) -> torch.Tensor:
    """bf16 RMSNorm(x) * w over the full row of x [M, D], then RoPE of every head's (even, odd)
    pairs by rope [M, head_dim // 2, 2] (cos, sin) fp32 when given."""
    _req(x, torch.bfloat16, "x")
    _req(w, torch.bfloat16, "w")
    if rope is not None:
        _req(rope, torch.float32, "rope")
    M, D = x.shape
    out = torch.empty_like(x) if out is None else out
    check(lib().fw_rms_rope(ptr(x), M, D, float(eps), ptr(w), ptr(rope), head_dim, ptr(out), stream_ptr()),
          "rms_rope")
    return out
