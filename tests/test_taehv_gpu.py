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


def test_prefix_cache_with_tinyvae_matches_serving_from_scratch():
    """PrefixCache over a session with the real decoder: the frames served with checkpoint
    sharing (a bounded pool, so restores, evictions and latent replays through the decoder all
    happen) equal serving every request from scratch, bit for bit."""
    from fastworld_b200.config import SMALL
    from fastworld_b200.prefix_cache import PrefixCache
    from fastworld_b200.static import B200StaticMG
    from fastworld_b200.vae import TAEW2_1, TinyVAE
    from fastworld_b200.weights import synthetic_state_dict
    S = B200StaticMG(SMALL, synthetic_state_dict(SMALL, 0))
    S.add_image("img0", seed=5, max_chunks=8)
    S.capture(warmup=1)
    vae = TinyVAE("cuda:0", cfg=TAEW2_1, seed=1)
    trunk = [("img0", (k, c)) for k, c in zip("wwsadw", "uijkli")]
    paths = [trunk, trunk[:4] + [("img0", ("q", "u"))] * 2, trunk[:2] + [("img0", ("d", "j"))], trunk[:5]]
    served = []
    for every, bound in ((None, None), (2, 1)):
        cache = PrefixCache(S, vae, every=every, max_checkpoints=bound)
        got = []
        for p in paths:
            frames, _ = cache.serve(p)
            got.append(frames)
        served.append(got)
        if every:
            assert cache.n_evicted > 0
    for a, b in zip(*served):
        assert len(a) == len(b)
        for fa, fb in zip(a, b):
            assert torch.equal(fa, fb)
    assert served[0][0][0].shape[0] == TAEW2_1.frames_out - TAEW2_1.trim
    assert vae.device_status() == 0
    S.graphs = {}
