"""tcgen05 GEMM parity against an fp32 PyTorch reference of the same op (bf16 inputs).

Covers the tile widths (64/128/224/256 and the 256 x 256 CTA-pair tile, tile_n 512), M/N/K tails (TMA zero fill + masked epilogue), every
epilogue (bias, GELU-tanh, GELU-erf, fp32 store, gated fp32 residual) and the MG2 shapes.
Tolerance: rel-L2 <= 6e-3 and max-abs <= 3e-2 * max|ref| (bf16 output rounding is 2^-9).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def _data(M, N, K, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    bias = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    return a, b, bias


SHAPES = [(128, 256, 64, 256), (300, 512, 200, 256), (2640, 1536, 1536, 256), (257, 1280, 1280, 128),
          (2640, 64, 1536, 64), (200, 384, 136, 128), (2640, 4608, 1536, 256), (2640, 1536, 8960, 256),
          (96, 96, 72, 64),
          # CTA pair (cta_group::2): tails in M, N and K, one and several tiles per pair
          (256, 256, 64, 512), (300, 544, 200, 512), (2640, 1536, 1536, 512), (4680, 7680, 512, 512)]


@pytest.mark.parametrize("M,N,K,tile", SHAPES)
def test_gemm_bias(M, N, K, tile):
    from fastworld_b200 import ops
    a, b, bias = _data(M, N, K)
    out = ops.gemm(a, b, bias, "none", tile)
    ref = a.float() @ b.float().t() + bias.float()
    torch.cuda.synchronize()
    assert _rel(out, ref) < 6e-3
    assert float((out.float() - ref).abs().max()) <= 3e-2 * float(ref.abs().max())


@pytest.mark.parametrize("epi", ["gelu_tanh", "gelu_erf", "f32"])
def test_gemm_epilogues(epi):
    from fastworld_b200 import ops
    a, b, bias = _data(640, 768, 512, seed=1)
    out = ops.gemm(a, b, bias, epi)
    ref = a.float() @ b.float().t() + bias.float()
    if epi == "gelu_tanh":
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    elif epi == "gelu_erf":
        ref = torch.nn.functional.gelu(ref)
    assert out.dtype == (torch.float32 if epi == "f32" else torch.bfloat16)
    assert _rel(out, ref) < (1e-5 if epi == "f32" else 6e-3)


@pytest.mark.parametrize("M,N,K,rpf", [
    (2640, 1536, 1536, 880),   # MG2 o-projection: 224-wide tiles (21 x 7 = 147 on 148 SMs)
    (2640, 1536, 8960, 880),   # MG2 ffn.2
    (300, 480, 200, 100),      # 224-wide, last column tile 32 of 224 valid, M and K tails
    (6032, 1536, 256, 1508),   # LingBot rows: 256-wide tiles (two full waves)
])
def test_gemm_residual_gate(M, N, K, rpf):
    from fastworld_b200 import ops
    a, b, bias = _data(M, N, K, seed=2)
    g = torch.Generator(device="cuda").manual_seed(3)
    resid = torch.randn(M, N, device="cuda", generator=g)
    gate = torch.randn((M + rpf - 1) // rpf, N, device="cuda", generator=g)
    ref = resid + gate.repeat_interleave(rpf, 0)[:M] * (a.float() @ b.float().t() + bias.float())
    ops.gemm_resid_(resid, a, b, bias, gate, rpf)
    assert _rel(resid, ref) < 1e-5


def test_gemm_tile_224_f32_and_limits():
    """The 224-wide tile with the fp32-output epilogue agrees with the 256-wide one (same K order
    per element); bf16-output epilogues are refused at that width."""
    from fastworld_b200 import ops
    a, b, bias = _data(2640, 1536, 1536, seed=7)
    x = ops.gemm(a, b, bias, "f32", 224)
    y = ops.gemm(a, b, bias, "f32", 256)
    torch.cuda.synchronize()
    assert _rel(x, y) < 1e-6
    with pytest.raises(RuntimeError):
        ops.gemm(a, b, bias, "none", 224)


def test_gemm_deterministic():
    from fastworld_b200 import ops
    a, b, bias = _data(2640, 1536, 1536, seed=4)
    x = ops.gemm(a, b, bias)
    y = ops.gemm(a, b, bias)
    assert torch.equal(x, y)


@pytest.mark.parametrize("epi", ["gelu_tanh", "f32"])
def test_gemm_pair_epilogues(epi):
    """The CTA-pair kernel's epilogues agree bitwise with the one-CTA kernel's (same fp32
    accumulation order per output element: K blocks in order)."""
    from fastworld_b200 import ops
    a, b, bias = _data(700, 768, 512, seed=5)
    one = ops.gemm(a, b, bias, epi, 256)
    two = ops.gemm(a, b, bias, epi, 512)
    torch.cuda.synchronize()
    assert _rel(two, one) < 1e-6


def test_gemm_pair_e4m3_matches_one_cta():
    from fastworld_b200 import ops
    a, b, bias = _data(2640, 1536, 1536, seed=6)
    a8, sa = ops.quant_e4m3(a)
    b8, sw = ops.quant_e4m3(b)
    one = ops.gemm_e4m3(a8, sa, b8, sw, bias, "none", 256)
    two = ops.gemm_e4m3(a8, sa, b8, sw, bias, "none", 512)
    torch.cuda.synchronize()
    assert torch.equal(one, two)
