"""16-chunk autoregressive drift on the GPU at test size: the engine and the oracle each run on
their own state over 16 chunks of one path (same inputs); the latent error must stay within
the single-chunk tolerance (rel-L2 <= 3e-2) all the way.  The full-size (MG2) report comes from
tests/drift_report.py."""
import pytest

from fastworld_b200.config import SMALL

pytestmark = pytest.mark.gpu


def test_sixteen_chunks_stay_within_tolerance():
    from drift_report import make_path
    from oracle.mg2_oracle import Oracle
    from fastworld_b200.prep import action_windows, synthetic_image
    from fastworld_b200.static import B200StaticMG
    from fastworld_b200.weights import synthetic_state_dict
    cfg = SMALL
    sd = synthetic_state_dict(cfg, 0)
    S = B200StaticMG(cfg, sd)
    img = synthetic_image(cfg, 5, 17)
    S.add_image("img0", img)
    path = make_path(16)
    orc = Oracle(cfg, sd)
    st = orc.new_state()
    errs = []
    for k in range(16):
        S._prep(path, k)
        x_in, noise = S.x_in.cpu(), [n.cpu() for n in S.noise]
        S._chunk(k == 0)
        kc, gm = action_windows(cfg, path, k)
        s = cfg.frames * k
        inp = {"cc": img["cond_concat"][0, :, s:s + cfg.frames].float(), "vis": img["visual_context"][0].float(),
               "gm": gm, "kc": kc, "k": k}
        ref = orc.chunk(st, x_in[0].float(), [n.float() for n in noise], inp, k == 0)
        out = S.out[0].float().cpu()
        errs.append(float((out - ref).norm() / ref.norm()))
    print("latent rel-L2 per chunk:", " ".join(f"{e:.2e}" for e in errs))
    assert S.device_status()[0] == 0
    assert max(errs) < 3e-2, errs
