"""LingBot runtime, host side (no GPU): the KV plans against the reference's own function, the
engine's tensor table and roll count, and the oracle's window bookkeeping."""
import ctypes
import json
import os

import torch

from fastworld_b200.lingbot import (LINGBOT, LINGBOT_SMALL, chunk_plans, eager_plans, flow_schedule, make_config,
                                    pack_weights, synthetic_inputs, synthetic_state_dict)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "lingbot_plans.json")


def _tup(p):
    roll, woff, klen = p
    return (tuple(roll) if roll is not None else None, woff, klen)


def test_plans_match_the_reference():
    """``tests/golden/lingbot_plans.json`` holds the reference's eager_plans output (static.py:30-46)."""
    for case in json.load(open(GOLDEN)):
        got = eager_plans(case["n"], case["C"], case["W"], case["S"])
        assert [_tup(p) for p in got] == [_tup(p) for p in case["plans"]], case


def test_chunk_plans_and_the_five_distinct_plans():
    """The reference records one graph per distinct plan: 5 for C = 4, a window of 18 frames and a
    sink of 6 (static.py:1-13); chunk 3 ends with the roll [8:16] -> [6:14], steady chunks with
    [10:18] -> [6:14]."""
    pl = chunk_plans(16, 4)
    assert pl[:5] == [(0, 4, None), (4, 8, None), (8, 12, None), (12, 16, (8, 6, 8)), (14, 18, (10, 6, 8))]
    assert len(set(pl)) == 5 and all(p == pl[4] for p in pl[4:])


def test_schedule_constants():
    t, sig_x0, a, s = flow_schedule()
    assert t[0] == 1000.0 and all(t[i] > t[i + 1] for i in range(3))
    assert all(abs(x - ti / 1000.0) < 2e-3 for x, ti in zip(sig_x0, t))
    assert all(abs(ai + si - 1.0) < 1e-6 for ai, si in zip(a, s))


def test_capi_tensor_table_and_roll_pieces():
    from fastworld_b200 import _lib
    L = _lib.lib()
    for cfg, pieces in ((LINGBOT, 4), (LINGBOT_SMALL, 4)):
        c = make_config(cfg)
        h = ctypes.c_void_p()
        assert L.fw_lb_create(ctypes.byref(c), ctypes.byref(h)) == 0
        try:
            infos = {}
            for i in range(L.fw_lb_tensor_count(h)):
                inf = _lib.FwTensorInfo()
                assert L.fw_lb_tensor_info_at(h, i, ctypes.byref(inf)) == 0
                infos[inf.name.decode()] = (inf.kind, tuple(inf.shape[j] for j in range(inf.ndim)))
            assert infos["K.0"][1] == (cfg.kv_tokens, cfg.dim)
            assert infos["x_in"][1] == (16, cfg.chunk, cfg.lat_h, cfg.lat_w)
            weights = {k for k, v in infos.items() if v[0] == _lib.KIND_WEIGHT}
            if cfg is LINGBOT_SMALL:
                pk = pack_weights(cfg, synthetic_state_dict(cfg, 0))
                assert weights == set(pk)
                assert all(tuple(pk[k].shape) == infos[k][1] for k in weights)
            assert L.fw_lb_roll_pieces(h) == pieces
            assert L.fw_lb_finalize(h) == -5   # nothing bound
        finally:
            L.fw_lb_destroy(h)
    bad = make_config(LINGBOT_SMALL)
    bad.kv_frames = 2
    assert L.fw_lb_create(ctypes.byref(bad), ctypes.byref(ctypes.c_void_p())) == -2


def test_oracle_window_keeps_the_sink_and_rolls_the_rest():
    """The oracle's window: the sink frames (0-5, written by chunks 0 and 1) never change, and
    the end-of-chunk roll moves frames [src, src + n) to [dst, dst + n) (static.py:257-264)."""
    from oracle.lingbot_oracle import LingbotOracle
    cfg = LINGBOT_SMALL.replace(layers=1)
    orc = LingbotOracle(cfg, synthetic_state_dict(cfg, 0))
    I = synthetic_inputs(cfg, 6, seed=2, text_tokens=8)
    orc.set_prompt(I.context)
    st = orc.new_state()
    plans = chunk_plans(6, cfg.chunk)
    Ft, C = cfg.frame_tokens, cfg.chunk
    g = torch.Generator().manual_seed(0)
    sink = None
    for k in range(6):
        s = C * k
        noise = [torch.randn(16, C, cfg.lat_h, cfg.lat_w, generator=g) for _ in range(3)]
        before = st["K"][0].clone()
        woff, klen, roll = plans[k]
        orc.chunk(st, k, plans[k], I.noise[:, s:s + C], I.y[:, s:s + C], I.plucker[0, :, s:s + C], noise)
        K = st["K"][0]
        if roll is not None:
            src, dst, n = roll
            # frames [src, woff) held older chunks' keys before this chunk; they now sit at dst
            assert torch.equal(K[dst * Ft:(dst + woff - src) * Ft], before[src * Ft:woff * Ft])
        if k == 1:
            sink = K[:cfg.sink * Ft].clone()
        if k > 1:
            assert torch.equal(K[:cfg.sink * Ft], sink)
        live = klen if roll is None else roll[1] + roll[2]
        assert bool((K[:live * Ft].reshape(live, -1).abs().sum(1) > 0).all())
