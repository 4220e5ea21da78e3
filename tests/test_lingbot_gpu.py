"""LingBot runtime on the GPU against the CPU oracle, over enough chunks to cover every plan of a
window of 18 frames with a 6-frame sink (chunks 0-2 without a roll, chunk 3's roll [8:16] ->
[6:14], the steady roll [10:18] -> [6:14]).  Same weights, inputs and renoising draws on both
sides; bounds per chunk on the x0 latent and on every layer's KV window: rel-L2 <= 1e-2 and
max-abs <= 1e-2 (relative to the largest reference magnitude); measured 2.3e-3 / 2.5e-3 / 4.6e-3
(small model) and 2.1e-3 / 2.5e-3 / 4.5e-3 (the reference's widths, 2 blocks)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

REL, ABS = 1e-2, 1e-2


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def _mx(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30))


def test_lingbot_small_matches_oracle_over_all_plans():
    from fastworld_b200.lingbot import LINGBOT_SMALL, B200StaticLingbot, synthetic_inputs, synthetic_state_dict
    from oracle.lingbot_oracle import LingbotOracle
    cfg = LINGBOT_SMALL
    n = 7
    sd = synthetic_state_dict(cfg, 0)
    I = synthetic_inputs(cfg, n, seed=3, text_tokens=10)
    S = B200StaticLingbot(cfg, sd, device="cuda:0")
    S.set_session(I)
    S.capture()
    orc = LingbotOracle(cfg, sd)
    orc.set_prompt(I.context)
    st = orc.new_state()
    errs = []
    for k in range(n):
        S._prep(k)
        noise = [t.cpu() for t in S.noise]
        S.graph.replay()
        got = S.out.clone()
        torch.cuda.synchronize()
        s = cfg.chunk * k
        ref = orc.chunk(st, k, S.plans[k], I.noise[:, s:s + cfg.chunk], I.y[:, s:s + cfg.chunk],
                        I.plucker[0, :, s:s + cfg.chunk], noise)
        e = (_rel(got.cpu(), ref), _mx(got.cpu(), ref))
        kv = max(max(_rel(S.K[i].cpu(), st["K"][i].reshape(cfg.kv_tokens, -1)),
                     _rel(S.V[i].cpu(), st["V"][i].reshape(cfg.kv_tokens, -1))) for i in range(cfg.layers))
        errs.append((k, e, kv))
        assert e[0] <= REL and e[1] <= ABS and kv <= REL, f"chunk {k}: x0 {e}, KV {kv:.3e}"
    print("lingbot_small x0 rel-L2 / max-abs and max KV rel-L2 per chunk:", errs)
    assert S.device_status() == 0


def test_lingbot_width_two_layers_matches_oracle():
    """The reference's widths (dim 1536, 12 heads, FFN 8960, 512-token prompt of width 4096,
    384 camera channels) with 2 blocks and a 16 x 32 latent frame (512 tokens per chunk, a
    2304-key window), 7 chunks over every plan; same bounds as the small model."""
    from fastworld_b200.lingbot import LINGBOT, B200StaticLingbot, synthetic_inputs, synthetic_state_dict
    from oracle.lingbot_oracle import LingbotOracle
    cfg = LINGBOT.replace(layers=2, lat_h=16, lat_w=32)
    n = 7
    sd = synthetic_state_dict(cfg, 1)
    I = synthetic_inputs(cfg, n, seed=5, text_tokens=40)
    S = B200StaticLingbot(cfg, sd, device="cuda:0")
    S.set_session(I)
    S.capture()
    orc = LingbotOracle(cfg, sd)
    orc.set_prompt(I.context)
    st = orc.new_state()
    errs = []
    for k in range(n):
        S._prep(k)
        noise = [t.cpu() for t in S.noise]
        S.graph.replay()
        got = S.out.clone()
        torch.cuda.synchronize()
        s = cfg.chunk * k
        ref = orc.chunk(st, k, S.plans[k], I.noise[:, s:s + cfg.chunk], I.y[:, s:s + cfg.chunk],
                        I.plucker[0, :, s:s + cfg.chunk], noise)
        e = (_rel(got.cpu(), ref), _mx(got.cpu(), ref))
        kv = max(max(_rel(S.K[i].cpu(), st["K"][i].reshape(cfg.kv_tokens, -1)),
                     _rel(S.V[i].cpu(), st["V"][i].reshape(cfg.kv_tokens, -1))) for i in range(cfg.layers))
        errs.append((k, e, kv))
        assert e[0] <= REL and e[1] <= ABS and kv <= REL, f"chunk {k}: x0 {e}, KV {kv:.3e}"
    print("lingbot width x0 rel-L2 / max-abs and max KV rel-L2 per chunk:", errs)
    assert S.device_status() == 0


def test_lingbot_graph_equals_eager_and_state_restores():
    """One graph for every plan gives the eager launches' bytes; a saved state (live window prefix
    + generator) reproduces the following chunk bit for bit (static.py:307-316)."""
    from fastworld_b200.lingbot import LINGBOT_SMALL, B200StaticLingbot, synthetic_inputs
    cfg = LINGBOT_SMALL
    I = synthetic_inputs(cfg, 7, seed=4, text_tokens=6)
    S = B200StaticLingbot(cfg, device="cuda:0", seed=1)
    S.set_session(I)
    eager = [S.gen_chunk(k, graph=False) for k in range(6)]
    S.reset()
    S.capture()
    graph = [S.gen_chunk(k, graph=True) for k in range(4)]
    st = S.state()
    a = [S.gen_chunk(k) for k in (4, 5)]
    S.load(st)
    b = [S.gen_chunk(k) for k in (4, 5)]
    torch.cuda.synchronize()
    for x, y in zip(eager[:4], graph):
        assert torch.equal(x, y)
    for x, y, z in zip(a, b, eager[4:]):
        assert torch.equal(x, y) and torch.equal(x, z)
    assert S.state_bytes() == 2 * cfg.layers * cfg.kv_tokens * cfg.dim * 2 * 14 // 18
