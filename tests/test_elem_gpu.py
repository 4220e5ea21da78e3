"""The memory-bound row kernels against plain PyTorch fp32 references of the same ops:
LayerNorm (fp32 residual in, bf16 out) with the adaLN modulate (norm1 / norm2, static.py:206,
224) and with the affine (norm3, static.py:221), and the q/k RMSNorm over the full width
followed by RoPE (static.py:207-212, 130-133).  Tolerance: bf16 output rounding, rel-L2 <= 4e-3."""
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 4e-3


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.parametrize("M,D", [(2640, 1536), (4680, 5120), (257, 1280), (5, 256)])
def test_layernorm_modulate_and_affine(M, D):
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(M + D)
    x = torch.randn(M, D, device="cuda", generator=g) * 3 + 0.5
    shift, scale = torch.randn(D, device="cuda", generator=g) * 0.3, torch.randn(D, device="cuda", generator=g) * 0.3
    ref = torch.nn.functional.layer_norm(x, (D,), eps=1e-6) * (1 + scale) + shift
    assert rel(ops.layernorm(x, 1e-6, shift=shift, scale=scale), ref) < TOL
    w, b = (torch.randn(D, device="cuda", generator=g) * 0.5 + 1).bfloat16(), torch.randn(D, device="cuda",
                                                                                            generator=g).bfloat16()
    ref = torch.nn.functional.layer_norm(x, (D,), w.float(), b.float(), eps=1e-6)
    assert rel(ops.layernorm(x, 1e-6, w=w, b=b), ref) < TOL
    ref = torch.nn.functional.layer_norm(x, (D,), eps=1e-6)
    assert rel(ops.layernorm(x, 1e-6), ref) < TOL


@pytest.mark.parametrize("M,D", [(2640, 1536), (4680, 640), (100, 384)])
def test_rms_rope(M, D):
    from fastworld_b200 import ops
    hd = 128
    g = torch.Generator(device="cuda").manual_seed(M * 7 + D)
    x = (torch.randn(M, D, device="cuda", generator=g) * 2).bfloat16()
    w = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    ang = torch.rand(M, hd // 2, device="cuda", generator=g) * 6.3
    rope = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    yc = torch.view_as_complex(y.view(M, D // hd, hd // 2, 2).contiguous())
    ref = torch.view_as_real(yc * torch.polar(torch.ones_like(ang), ang)[:, None]).reshape(M, D)
    assert rel(ops.rms_rope(x, w, rope, hd), ref) < TOL
    assert rel(ops.rms_rope(x, w, None, hd), y) < TOL
