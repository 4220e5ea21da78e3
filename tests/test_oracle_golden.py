"""Pin the CPU oracle to the reference's own StaticMG code (fixtures from make_golden.py).

The fixture was produced by running ``fastworld/models/mg2/static.py`` (``_prep``, ``_net``,
``_chunk``, ``gen_chunk``, ``prefill``, ``state``/``load``) unmodified on the CPU in fp32 with
stand-in layers; here the independent functional oracle must reproduce it to fp32 precision,
and the product's host-side prep (action windows, noise order, RoPE table) must match exactly.
"""
import copy
import os

import pytest
import torch

from fastworld_b200.config import PRESETS
from fastworld_b200.prep import action_windows, draw_noise, path_seed, synthetic_image
from fastworld_b200.weights import synthetic_state_dict
from oracle.mg2_oracle import Oracle, rope_table

GOLD = os.path.join(os.path.dirname(__file__), "golden", "tiny_ref.pt")


def _close(sample, t, rtol):
    flat = t.reshape(-1).double()
    got = flat[sample["idx"]]
    ref = sample["val"].double()
    err = (got - ref).norm() / ref.norm().clamp_min(1e-30)
    assert err < rtol, f"rel-L2 {err:.3e} >= {rtol}"
    assert abs(float(flat.sum()) - sample["sum"]) <= rtol * (1 + abs(sample["sum"])) * 10
    assert abs(float((flat * flat).sum()) - sample["sumsq"]) <= rtol * sample["sumsq"] * 10


@pytest.fixture(scope="module")
def gold():
    return torch.load(GOLD, weights_only=False)


@pytest.fixture(scope="module")
def setup(gold):
    cfg = PRESETS[gold["config"]]
    sd = synthetic_state_dict(cfg, gold["seed"])
    img = synthetic_image(cfg, gold["img_seed"], 8)
    return cfg, Oracle(cfg, sd, round_interface=False), img


def _inputs(cfg, img, path, k):
    kc, gm = action_windows(cfg, path, k)
    s = cfg.frames * k
    return {"cc": img["cond_concat"][0, :, s:s + cfg.frames], "vis": img["visual_context"][0],
            "gm": gm, "kc": kc, "k": k}


def test_prep_matches_reference(gold, setup):
    cfg, orc, img = setup
    path = gold["path"]
    for ch in gold["chunks"]:
        k = ch["k"]
        assert path_seed(path[:k + 1]) == ch["path_seed"]
        kc, gm = action_windows(cfg, path, k)
        assert torch.equal(kc.float(), ch["kc"]), k
        assert torch.equal(gm.float(), ch["gm"]), k
        fi = torch.view_as_real(rope_table(cfg, k, orc.freqs)).reshape(-1)
        assert torch.allclose(fi[ch["fi"]["idx"]].float(), ch["fi"]["val"], atol=1e-7)
        nz = draw_noise(cfg, path, k)
        _close(ch["x_in"], nz[0].float(), 1e-7)
        for s, t in zip(ch["noise"], nz[1:]):
            _close(s, t.float(), 1e-7)


def test_chunks_state_branch_prefill_match_reference(gold, setup):
    cfg, orc, img = setup
    path = gold["path"]
    st = orc.new_state()
    for ch in gold["chunks"]:
        k = ch["k"]
        nz = draw_noise(cfg, path, k)
        out = orc.chunk(st, nz[0][0].float(), [t.float() for t in nz[1:]], _inputs(cfg, img, path, k), k == 0)
        _close(ch["out"], out[None], 2e-4)
    g = gold["state"]
    for i in range(cfg.layers):
        _close(g["hk"][i], st["hk"][i], 2e-4)
        _close(g["hv"][i], st["hv"][i], 2e-4)
    for nm in ("mk", "mv", "kk", "kv"):
        for i, s in g[nm].items():
            _close(s, st[nm][i], 2e-4)
    saved = copy.deepcopy(st)
    alt = path[:3] + [("img0", ("s", "k"))]
    nz = draw_noise(cfg, alt, 3)
    orc.chunk(st, nz[0][0].float(), [t.float() for t in nz[1:]], _inputs(cfg, img, alt, 3), False)
    st = copy.deepcopy(saved)
    nz = draw_noise(cfg, path, 3)
    out = orc.chunk(st, nz[0][0].float(), [t.float() for t in nz[1:]], _inputs(cfg, img, path, 3), False)
    _close(gold["branch_out"], out[None], 2e-4)
    st = copy.deepcopy(saved)
    orc.prefill(st, out, _inputs(cfg, img, path, 3), False)
    _close(gold["prefill_hk0"], st["hk"][0], 2e-4)
