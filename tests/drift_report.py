"""16-chunk drift of the sm_100a engine against the fp32 CPU oracle (north_star: "multi-chunk
drift over 16 chunks must be reported").

Two steps, so the slow CPU side can run on any host:

    python tests/drift_report.py run --config mg2 --chunks 16 --out drift_mg2.pt   # GPU
    python tests/drift_report.py compare drift_mg2.pt [--threads N]                # CPU

``run`` plays chunks 0..N-1 of one seeded path through ``B200StaticMG`` (each chunk on the
engine's own state) and saves, per chunk, the inputs drawn on the device (x_in, noise), the
output latent and per-layer fp64 sums / sums of squares of the history K/V.  ``compare``
replays the same inputs through the oracle on its own state and prints one JSON line per
chunk plus a summary: rel-L2 of the latent and the largest per-layer relative difference of
the history sums of squares.  Both sides use the same seeded weights, image and actions.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from fastworld_b200.config import PRESETS  # noqa: E402
from fastworld_b200.prep import action_windows, synthetic_image  # noqa: E402
from fastworld_b200.weights import synthetic_state_dict  # noqa: E402

KEYS = ("w", "s", "a", "d", "q")
CAMS = ("i", "k", "j", "l", "u")


def make_path(n):
    g = torch.Generator().manual_seed(11)
    return [("img0", (KEYS[int(torch.randint(5, (1,), generator=g))], CAMS[int(torch.randint(5, (1,), generator=g))]))
            for _ in range(n)]


def hist_sums(hk, hv):
    return torch.tensor([[t.double().sum().item(), t.double().pow(2).sum().item()] for t in list(hk) + list(hv)])


def run(a):
    from fastworld_b200.static import B200StaticMG
    cfg = PRESETS[a.config]
    sd = synthetic_state_dict(cfg, 0)
    S = B200StaticMG(cfg, sd)
    img = synthetic_image(cfg, 5, a.chunks + 1)
    S.add_image("img0", img)
    path = make_path(a.chunks)
    rec = []
    for k in range(a.chunks):
        S._prep(path, k)
        x_in, noise = S.x_in.cpu().clone(), [n.cpu().clone() for n in S.noise]
        S._chunk(k == 0)
        torch.cuda.synchronize()
        rec.append({"x_in": x_in, "noise": noise, "out": S.out.cpu().clone(),
                    "hist": hist_sums([h[0] for h in S.hk], [h[0] for h in S.hv])})
    assert S.device_status()[0] == 0
    os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
    torch.save({"config": a.config, "chunks": a.chunks, "rec": rec}, a.out)
    print(f"saved {a.chunks} chunks to {a.out}")


def compare(a):
    from oracle.mg2_oracle import Oracle
    if a.threads:
        torch.set_num_threads(a.threads)
    d = torch.load(a.file)
    cfg = PRESETS[d["config"]]
    sd = synthetic_state_dict(cfg, 0)
    img = synthetic_image(cfg, 5, d["chunks"] + 1)
    path = make_path(d["chunks"])
    orc = Oracle(cfg, sd)
    st = orc.new_state()
    rows = []
    for k, r in enumerate(d["rec"]):
        kc, gm = action_windows(cfg, path, k)
        s = cfg.frames * k
        inp = {"cc": img["cond_concat"][0, :, s:s + cfg.frames].float(), "vis": img["visual_context"][0].float(),
               "gm": gm, "kc": kc, "k": k}
        with torch.no_grad():
            ref = orc.chunk(st, r["x_in"][0].float(), [n.float() for n in r["noise"]], inp, k == 0)
        out = r["out"][0].float()
        hs = hist_sums(st["hk"], st["hv"])
        row = {"chunk": k, "latent_rel_l2": float((out - ref).norm() / ref.norm()),
               "latent_max_abs": float((out - ref).abs().max()),
               "hist_sumsq_rel_max": float(((r["hist"][:, 1] - hs[:, 1]).abs() / hs[:, 1].abs().clamp_min(1e-30)).max())}
        rows.append(row)
        print(json.dumps(row), flush=True)
    print("DRIFT_SUMMARY " + json.dumps({"config": d["config"], "chunks": len(rows),
                                         "latent_rel_l2_first": rows[0]["latent_rel_l2"],
                                         "latent_rel_l2_last": rows[-1]["latent_rel_l2"],
                                         "latent_rel_l2_max": max(x["latent_rel_l2"] for x in rows),
                                         "hist_sumsq_rel_max": max(x["hist_sumsq_rel_max"] for x in rows)}))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--config", default="mg2")
    r.add_argument("--chunks", type=int, default=16)
    r.add_argument("--out", default="drift_mg2.pt")
    c = sub.add_parser("compare")
    c.add_argument("file")
    c.add_argument("--threads", type=int, default=0)
    a = ap.parse_args()
    run(a) if a.cmd == "run" else compare(a)
