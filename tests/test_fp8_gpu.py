"""e4m3 variant: quantisation, the kind::f8f6f4 GEMM, and the engine.

* the row quantiser matches torch's float8_e4m3fn conversion of x / (absmax / 448) bit for bit;
* the e4m3 GEMM matches an fp32 reference of the same dequantised operands (rel-L2 <= 6e-3);
* the engine with e4m3 FFN linears ("fp8_ffn": ffn.0 and ffn.2, 65 % of the block's GEMM
  flops) against the bf16 engine on the same weights and inputs: latent and every layer's
  history K/V within BASELINE's rel-L2 <= 2e-2, at MG2 width (2 layers) and at full depth
  (30 layers), chunk 0 and a steady chunk;
* the engine with every block linear in e4m3 ("fp8"): rel-L2 is bounded at the measured level
  (3.9e-2 at 2 layers); BASELINE's 2e-2 is not met and is kept as a strict expected failure.
  E4m3 has 3 mantissa bits: rounding both operands adds 3.3-3.8 % rel-L2 to every GEMM output
  whatever the scale granularity (per token / per channel, 1 x 128 or 1 x 32 blocks, measured
  on the CPU), and the attention-side and action-module linears carry that noise into the
  latent (5.0e-2 at 30 layers on the CPU emulation, 5.8-6.5e-2 measured on a B200).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _deq(q, sc):
    return q.view(torch.float8_e4m3fn).float() * sc[:, None]


def test_quant_matches_torch():
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(300, 1536, device="cuda", generator=g) * torch.rand(300, 1, device="cuda", generator=g) * 5).to(
        torch.bfloat16)
    x[7] = 0
    q, sc = ops.quant_e4m3(x)
    amax = x.float().abs().amax(1)
    ref_sc = torch.where(amax > 0, amax / 448, torch.ones_like(amax))
    assert torch.allclose(sc, ref_sc, rtol=1e-6, atol=0)
    ref = (x.float() / ref_sc[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    assert (q != ref).sum().item() == 0


@pytest.mark.parametrize("M,N,K,tile", [(2640, 1536, 1536, 256), (2640, 8960, 1536, 256), (2640, 1536, 8960, 256),
                                        (300, 384, 272, 128), (257, 1024, 1024, 64)])
def test_gemm_e4m3(M, N, K, tile):
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    bias = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    a8, sa = ops.quant_e4m3(a)
    b8, sw = ops.quant_e4m3(b)
    out = ops.gemm_e4m3(a8, sa, b8, sw, bias, "none", tile)
    ref = _deq(a8, sa) @ _deq(b8, sw).t() + bias.float()
    err = float((out.float() - ref).norm() / ref.norm())
    assert err < 6e-3, err
    # and the quantisation error of the whole product stays small against bf16
    full = a.float() @ b.float().t() + bias.float()
    assert float((out.float() - full).norm() / full.norm()) < 6e-2


def fp8_vs_bf16(cfg, linear, chunks=2, seed=3):
    """Latent and per-layer history K/V rel-L2 of the e4m3 engine against the bf16 engine."""
    from fastworld_b200.prep import synthetic_image
    from fastworld_b200.static import B200StaticMG
    from fastworld_b200.weights import synthetic_state_dict
    sd = synthetic_state_dict(cfg, seed)
    img = synthetic_image(cfg, 4, chunks + 1)
    path = [("img0", ("w", "u")), ("img0", ("a", "l")), ("img0", ("d", "i"))][:chunks]
    runs = {}
    for lin in ("bf16", linear):
        S = B200StaticMG(cfg.replace(linear=lin), sd)
        S.add_image("img0", img)
        outs = []
        for k in range(chunks):
            outs.append((S.gen_chunk(path, k, graph=False).float().cpu(), [h.float().cpu() for h in S.hk],
                         [v.float().cpu() for v in S.hv]))
        assert S.device_status()[0] == 0
        runs[lin] = outs
        del S
        torch.cuda.empty_cache()
    rel = lambda a, b: float((a - b).norm() / b.norm())  # noqa: E731
    errs = []
    for (o8, k8, v8), (o, k, v) in zip(runs[linear], runs["bf16"]):
        errs.append({"out": rel(o8, o), "hk": max(rel(a, b) for a, b in zip(k8, k)),
                     "hv": max(rel(a, b) for a, b in zip(v8, v))})
    print(cfg.name, linear, errs)
    return errs


def test_engine_fp8_ffn_meets_2e2_mg2_width():
    from fastworld_b200.config import MG2
    for e in fp8_vs_bf16(MG2.replace(name="mg2_2l", layers=2, action_blocks=(1,)), "fp8_ffn"):
        assert max(e.values()) <= 2e-2, e


def test_engine_fp8_ffn_meets_2e2_full_depth():
    from fastworld_b200.config import MG2
    for e in fp8_vs_bf16(MG2, "fp8_ffn"):
        assert max(e.values()) <= 2e-2, e


def test_engine_fp8_all_linears_measured_bound():
    from fastworld_b200.config import SMALL
    for e in fp8_vs_bf16(SMALL, "fp8"):
        assert e["out"] < 5e-2, e


@pytest.mark.xfail(strict=True, reason="every block linear in e4m3: 3-4 % rounding noise per GEMM; the "
                                      "latent differs from bf16 by 4-6.5e-2, above BASELINE's 2e-2")
def test_engine_fp8_all_linears_2e2_target():
    from fastworld_b200.config import MG2
    for e in fp8_vs_bf16(MG2.replace(name="mg2_2l", layers=2, action_blocks=(1,)), "fp8"):
        assert max(e.values()) <= 2e-2, e
