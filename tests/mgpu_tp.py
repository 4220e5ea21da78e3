"""Two-rank helper for tests/test_tp_gpu.py (run under torchrun, one process per GPU).

Both ranks build the same tensor-parallel session (SMALL_TP: 4 heads and FFN 1024 over 2 GPUs,
a 2-chunk history window) and play chunks 0-3, which covers no history, one filled slot, two
slots and the ring wrap-around.  Rank 0 checks the latents and its heads' history against the
CPU oracle and against the same session on one GPU; both ranks must produce identical latents.
The collectives run on the engine's peer-memory kernels (workspaces mapped over NVLink); the
same session with NCCL collectives must agree.  Then chunk 4 is replayed from a snapshot
through captured CUDA graphs."""
import datetime
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from fastworld_b200.config import SMALL_TP  # noqa: E402
from fastworld_b200.prep import synthetic_image  # noqa: E402
from fastworld_b200.static import B200StaticMG  # noqa: E402
from fastworld_b200.weights import synthetic_state_dict  # noqa: E402

PATH = [("img0", ("w", "u")), ("img0", ("a", "l")), ("img0", ("q", "i")), ("img0", ("d", "j")),
        ("img0", ("s", "k"))]


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def main():
    rank, local, world = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(local)
    torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    cfg = SMALL_TP
    sd = synthetic_state_dict(cfg, 0)
    img = synthetic_image(cfg, 5, 8)
    S = B200StaticMG(cfg, sd, device=f"cuda:{local}", tp_group=True)
    S.add_image("img0", img)
    outs, inputs = [], []
    for k in range(4):
        S._prep(PATH, k)
        inputs.append((S.x_in.cpu(), [n.cpu() for n in S.noise]))
        S._chunk(k == 0)
        outs.append(S.out.clone())
    torch.cuda.synchronize()
    status = S.device_status()
    hist = [h.cpu() for h in S.hk]          # after chunk 3: slots hold chunks 2 and 3
    snap = S.state()
    out4 = S.gen_chunk(PATH, 4, graph=False)
    S.load(snap)
    S.capture(warmup=1)
    out4g = S.gen_chunk(PATH, 4)
    torch.cuda.synchronize()
    # the same model with the collectives on NCCL instead of the peer-memory kernels
    S2 = B200StaticMG(cfg, sd, device=f"cuda:{local}", tp_group=True, tp_peers=False)
    S2.add_image("img0", img)
    e_nccl = [rel(S2.gen_chunk(PATH, k, graph=False), outs[k]) for k in range(4)]
    status2 = S2.device_status()
    del S2
    res = {"rank": rank, "status": status, "graph_vs_eager": rel(out4g, out4), "nccl_rel": e_nccl,
           "status_nccl": status2, "outs": [o.cpu() for o in outs], "hk": hist}
    allres = [None] * world
    torch.distributed.all_gather_object(allres, res)
    if rank == 0:
        from oracle.mg2_oracle import Oracle
        torch.set_num_threads(8)
        same = all(torch.equal(allres[0]["outs"][k], r["outs"][k]) for r in allres for k in range(4))
        orc = Oracle(cfg, sd)
        st = orc.new_state()
        e_orc = []
        for k in range(4):
            s = cfg.frames * k
            from fastworld_b200.prep import action_windows
            kc, gm = action_windows(cfg, PATH, k)
            inp = {"cc": img["cond_concat"][0, :, s:s + cfg.frames].float(), "vis": img["visual_context"][0].float(),
                   "gm": gm, "kc": kc, "k": k}
            x_in, noise = inputs[k]
            ref = orc.chunk(st, x_in[0].float(), [n.float() for n in noise], inp, k == 0)
            e_orc.append(rel(outs[k][0], ref))
        Hl = cfg.heads // world
        e_hist = max(rel(allres[r]["hk"][i][0], st["hk"][i][:, r * Hl:(r + 1) * Hl]) for r in range(world)
                     for i in range(cfg.layers))
        # the same session on one GPU
        S1 = B200StaticMG(cfg, sd, device=f"cuda:{local}")
        S1.add_image("img0", img)
        e_tp1 = [rel(outs[k], S1.gen_chunk(PATH, k, graph=False)) for k in range(4)]
        line = {"ranks_identical": same, "oracle_rel": e_orc, "hist_rel": e_hist, "tp1_rel": e_tp1,
                "graph_vs_eager": max(r["graph_vs_eager"] for r in allres),
                "nccl_rel": max(max(r["nccl_rel"]) for r in allres),
                "status": [r["status"] for r in allres] + [r["status_nccl"] for r in allres]}
        print("TP_RESULT " + json.dumps(line), flush=True)
    S.graphs = {}
    del S
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
