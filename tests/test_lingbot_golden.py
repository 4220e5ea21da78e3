"""The LingBot oracle against the reference's own StaticLingbot (``tests/golden/lingbot_ref.pt``,
made by ``tests/golden/make_golden_lingbot.py`` from the unmodified ``static.py`` on the CPU with
stand-in modules, all in fp32): 7 chunks covering every KV plan, the window after them, and a
state restore."""
import os

import torch

from fastworld_b200.lingbot import LINGBOT_SMALL, chunk_plans, synthetic_inputs, synthetic_state_dict

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "lingbot_ref.pt")


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


def _check_sample(t, s, tol):
    flat = t.reshape(-1).double()
    assert tuple(t.shape) == tuple(s["shape"])
    assert float((flat[s["idx"]].float() - s["val"]).abs().max()) <= tol * float(s["val"].abs().max())
    assert abs(float(flat.sum()) - s["sum"]) <= tol * (abs(s["sum"]) + s["sumsq"] ** 0.5)


def test_oracle_matches_reference_static_lingbot():
    from oracle.lingbot_oracle import LingbotOracle
    ref = torch.load(GOLDEN, weights_only=False)
    cfg = LINGBOT_SMALL.replace(text_len=ref["text_len"])
    sd = synthetic_state_dict(cfg, ref["seed"])
    I = synthetic_inputs(cfg, len(ref["chunks"]), seed=ref["input_seed"], text_tokens=ref["text_tokens"])
    orc = LingbotOracle(cfg, sd, round_bf16=False)
    orc.set_prompt(I.context.float())
    st = orc.new_state()
    plans = chunk_plans(16, cfg.chunk)
    g = torch.Generator().manual_seed(I.seed)
    C = cfg.chunk
    saved = None
    for rec in ref["chunks"]:
        k = rec["k"]
        assert tuple(tuple(x) if isinstance(x, (list, tuple)) else x for x in rec["plan"]) == plans[k]
        noise = [torch.randn((16, C, cfg.lat_h, cfg.lat_w), generator=g, dtype=torch.float32) for _ in range(3)]
        s = C * k
        x0 = orc.chunk(st, k, plans[k], I.noise[:, s:s + C], I.y[:, s:s + C], I.plucker[0, :, s:s + C].float(), noise)
        assert _rel(x0, rec["x0"]) < 1e-5, (k, _rel(x0, rec["x0"]))
        if k == 4:
            saved = ({n: [t.clone() for t in v] for n, v in st.items()}, g.get_state())
    live = ref["chunks"][-1]["live"] * cfg.frame_tokens
    for i in range(cfg.layers):
        _check_sample(st["K"][i][:live], ref["window"]["K"][i], 1e-5)
        _check_sample(st["V"][i][:live], ref["window"]["V"][i], 1e-5)
    # restore the state after chunk 4 and run chunk 5 again (static.py:307-316)
    st = {n: [t.clone() for t in v] for n, v in saved[0].items()}
    g.set_state(saved[1])
    noise = [torch.randn((16, C, cfg.lat_h, cfg.lat_w), generator=g, dtype=torch.float32) for _ in range(3)]
    x0 = orc.chunk(st, 5, plans[5], I.noise[:, 5 * C:6 * C], I.y[:, 5 * C:6 * C], I.plucker[0, :, 5 * C:6 * C].float(),
                   noise)
    assert _rel(x0, ref["branch_x0"]) < 1e-5
