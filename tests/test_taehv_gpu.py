"""TAEHV streaming decoder on the GPU against the CPU oracle (fp32), through ``TinyVAE``.

The engine stores activations in fp16 (the reference runs TAEHV in fp16) and accumulates in
fp32; the oracle is fp32 throughout on the same fp16 weights and the fp16-rounded latent.
Bounds per chunk on the [-1, 1] frames: rel-L2 <= 5e-3 and max-abs <= 5e-2.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

REL, ABS = 5e-3, 5e-2


def _lat(cfg, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(1, 16, cfg.lat_frames, cfg.lat_h, cfg.lat_w, device="cuda", generator=g).to(torch.bfloat16)


def _errs(got, ref):
    rel = float((got.float().cpu() - ref).norm() / ref.norm())
    mx = float((got.float().cpu() - ref).abs().max())
    return rel, mx


def _stream(cfg, chunks, seed=0):
    from fastworld_b200.vae import TinyVAE, synthetic_state_dict
    from oracle.taehv_oracle import TaehvOracle
    vae = TinyVAE("cuda:0", cfg=cfg, seed=seed)
    orc = TaehvOracle(cfg, synthetic_state_dict(cfg, seed))
    out = []
    for k in range(chunks):
        lat = _lat(cfg, 100 + k)
        got = vae.decode(lat)
        ref = orc.decode(lat.cpu().half().float())
        assert got.shape == ref.shape
        out.append(_errs(got, ref))
    assert vae.device_status() == 0
    return out


def test_small_stream_matches_oracle():
    from fastworld_b200.vae import TAEHV_SMALL
    errs = _stream(TAEHV_SMALL, 3)
    print("taehv_small rel-L2 / max-abs per chunk", errs)
    for rel, mx in errs:
        assert rel <= REL and mx <= ABS


def test_taew2_1_matches_oracle():
    """The reference's decoder shape: [1, 16, 3, 44, 80] -> 9, then 12 frames of 352 x 640."""
    from fastworld_b200.vae import TAEW2_1
    errs = _stream(TAEW2_1, 2)
    print("taew2_1 rel-L2 / max-abs per chunk", errs)
    for rel, mx in errs:
        assert rel <= REL and mx <= ABS


def test_graph_replay_equals_eager_and_state_restores():
    """Graph replay and eager launches give the same bytes; restoring a saved state and decoding
    the same latent again reproduces the branch bit for bit (vae.py:112-119)."""
    from fastworld_b200.vae import TAEHV_SMALL, TinyVAE
    cfg = TAEHV_SMALL
    vae = TinyVAE("cuda:0", cfg=cfg, seed=3)
    vae.decode(_lat(cfg, 1), graph=False)
    st = vae.state()
    a = vae.decode(_lat(cfg, 2), graph=False)
    b_next = vae.decode(_lat(cfg, 3), graph=False)
    vae.load(st)
    a2 = vae.decode(_lat(cfg, 2), graph=True)
    b2 = vae.decode(_lat(cfg, 3), graph=True)
    torch.cuda.synchronize()
    assert torch.equal(a, a2) and torch.equal(b_next, b2)
    assert vae.state_bytes() == cfg.state_bytes()
    vae.reset()
    first = vae.decode(_lat(cfg, 1))
    assert first.shape[0] == cfg.frames_out - cfg.trim
