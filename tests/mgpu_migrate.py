"""Two-rank helper for tests/test_multigpu_gpu.py (run under torchrun, one process per GPU).

Rank 0 plays chunks 0-1 of a path, snapshots, exports the snapshot by CUDA IPC and plays chunk 2.
Rank 1 builds the same session (same seeded weights), pulls rank 0's snapshot over NVLink with
the engine's copy kernel and plays chunk 2.  Both chunk-2 latents must be bitwise equal."""
import datetime
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from fastworld_b200 import migrate  # noqa: E402
from fastworld_b200.config import SMALL  # noqa: E402
from fastworld_b200.static import B200StaticMG  # noqa: E402
from fastworld_b200.weights import synthetic_state_dict  # noqa: E402


def main():
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    S = B200StaticMG(SMALL, synthetic_state_dict(SMALL, 0), device=f"cuda:{local}")
    S.add_image("img0", seed=3, max_chunks=4)
    path = [("img0", ("w", "u")), ("img0", ("a", "l")), ("img0", ("d", "k"))]
    desc = None
    if rank == 0:
        for k in range(2):
            S.gen_chunk(path, k, graph=False)
        snap = S.state()
        torch.cuda.synchronize()
        desc = migrate.export_blob(snap.blob)
    got = [None, None]
    torch.distributed.all_gather_object(got, desc)
    if rank == 1:
        migrate.migrate_state(S, got[0])
        torch.cuda.synchronize()
    out = S.gen_chunk(path, 2, graph=False).cpu()
    outs = [None, None]
    torch.distributed.all_gather_object(outs, out)
    if rank == 0:
        same = torch.equal(outs[0], outs[1])
        print("MIGRATE_BITWISE", same, flush=True)
        assert same
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
