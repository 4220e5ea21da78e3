"""shared-start explore workload over 1..8 GPUs (one process per GPU).

    python -m fastworld_b200.explore [--sessions 64] [--chunks 16] [--rewinds 6] [--every 2]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m fastworld_b200.explore

All sessions start from the same seeded image latent and diverge by seeded random keyboard /
mouse actions.  Session i is served by rank i % N through that rank's ``PrefixCache``
(fastworld/prefix_cache.py:35-92) over one ``B200StaticMG``: 16 chunks, a checkpoint every 2
chunks, then 6 random rewinds (restore the deepest checkpoint before a random chunk, replay,
and play 2 new chunks).  A final cross-GPU phase restores, on every rank, checkpoints held by
the next rank (its most recently used ones): the owner exports the snapshot buffer by CUDA IPC and the receiver pulls it with
the engine's copy kernel over NVLink, then plays 2 chunks from it.

Reports (rank 0, one JSON line): aggregate served frames per second (max-over-ranks wall time),
generated / replayed / cached chunk counts, and the bandwidth of checkpoint save (``state()``),
local restore (``load``) and cross-GPU restore (peer pull).  No collective runs on the data path;
only IPC handles and counters cross the host process group (gloo).
"""
from __future__ import annotations

import argparse
import json
import os
import random
import time

import torch

from .prefix_cache import PrefixCache

KEY_NAMES = ("w", "s", "a", "d", "q")
CAM_NAMES = ("i", "k", "j", "l", "u")


class NullDecoder:
    """Stand-in for the (out-of-scope) video decoder: a tiny data-dependent view of the latent."""

    def decode(self, lat):
        return lat[0, :3, :, ::11, ::20].permute(1, 0, 2, 3).float().clamp(-1, 1)

    def reset(self):
        pass

    def state(self):
        return None

    def load(self, st):
        pass


def make_paths(n_sessions: int, chunks: int, seed: int, img: str = "img0"):
    rng = random.Random(seed)
    return [[(img, (rng.choice(KEY_NAMES), rng.choice(CAM_NAMES))) for _ in range(chunks)]
            for _ in range(n_sessions)]


def rewinds(path, n: int, every: int, seed: int, tail: int = 2):
    """n branches of `path`: keep a prefix that ends on a random checkpoint, play `tail` new chunks."""
    rng = random.Random(seed)
    out = []
    ks = list(range(every, len(path), every))
    for _ in range(n):
        t = rng.choice(ks)
        out.append(path[:t] + [(path[0][0], (rng.choice(KEY_NAMES), rng.choice(CAM_NAMES))) for _ in range(tail)])
    return out


def sessions_of(rank: int, world: int, n: int):
    return [i for i in range(n) if i % world == rank]


def timed_ms(fn):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    r = fn()
    e1.record()
    torch.cuda.synchronize()
    return r, e0.elapsed_time(e1)


def run(S, rank: int, world: int, sessions: int = 64, chunks: int = 16, n_rewinds: int = 6, every: int = 2,
        migrations: int = 2, max_checkpoints=None, group=None, img: str = "img0"):
    """Serve this rank's share of the explore workload on session ``S`` (captured graphs) and
    return this rank's counters and bandwidths.  Collective over ``group`` when world > 1
    (IPC descriptors and a barrier only)."""
    from . import migrate
    cache = PrefixCache(S, NullDecoder(), every=every, max_checkpoints=max_checkpoints)
    paths = make_paths(sessions, chunks, seed=1, img=img)
    mine = sessions_of(rank, world, sessions)
    stats = {"generated": 0, "replayed": 0, "hit": 0, "frames": 0, "restored": 0}
    if world > 1:
        torch.distributed.barrier(group=group)
    torch.cuda.synchronize()
    t0 = time.time()
    for i in mine:
        for p in [paths[i]] + rewinds(paths[i], n_rewinds, every, seed=1000 + i):
            frames, st = cache.serve(p)
            for k in ("generated", "replayed", "hit", "restored"):
                stats[k] += st[k]
            stats["frames"] += 12 * len(p)
    torch.cuda.synchronize()
    t_local = time.time() - t0
    # checkpoint bandwidth on this GPU: save (state) and restore (load) of the full session state
    nbytes = S._blob.numel()
    snap = S.state()                     # allocate once; time the copy kernels alone
    torch.cuda.synchronize()
    _, save_ms = timed_ms(lambda: migrate.pull_local(snap.blob, S._blob))
    _, load_ms = timed_ms(lambda: S.load(snap))
    del snap
    # cross-GPU phase: restore checkpoints held by the next rank here and play 2 chunks from each
    mig = {"count": 0, "ms": 0.0, "bytes": 0}
    if world > 1:
        held = sorted(cache.pool.holders, key=lambda n: -n.slot.stamp)[:migrations]   # most recently used
        offers = [([c.key for c in node.lineage()], migrate.export_blob(node.slot.runtime_state.blob))
                  for node in held]
        got = [None] * world
        torch.distributed.all_gather_object(got, offers, group=group)
        torch.cuda.synchronize()
        t1 = time.time()
        for prefix, desc in got[(rank + 1) % world]:
            with migrate.PeerBuffer(desc, S._blob.device) as peer:
                _, ms = timed_ms(lambda: migrate.pull(S._blob, peer))
            mig["count"] += 1
            mig["ms"] += ms
            mig["bytes"] += nbytes
            p = list(prefix) + [(prefix[0][0], ("w", "u"))] * 2
            for k in range(len(prefix), len(prefix) + 2):
                S.gen_chunk(p, k)
                stats["generated"] += 1
                stats["frames"] += 12
        torch.cuda.synchronize()
        t_local += time.time() - t1
        torch.distributed.barrier(group=group)   # owners keep their snapshots alive until every pull is done
    return {"rank": rank, "time": t_local, **stats, "save_gbs": 2 * nbytes / save_ms / 1e6,
            "load_gbs": 2 * nbytes / load_ms / 1e6, "state_bytes": nbytes,
            "peer_restore_gbs": (2 * mig["bytes"] / mig["ms"] / 1e6) if mig["ms"] else None,
            "migrations": mig["count"], "checkpoints": cache.n_ckpt, "evicted": cache.n_evicted}


def summarize(allres, world: int, sessions: int, chunks: int, n_rewinds: int, every: int, config: str):
    """One result over every rank: frames served / slowest rank's time, summed counters."""
    tmax = max(r["time"] for r in allres)
    keys = ("generated", "replayed", "hit", "frames", "restored", "migrations", "checkpoints", "evicted")
    tot = {k: sum(r[k] for r in allres) for k in keys}
    return {"workload": "explore (BASELINE configs[3])", "config": config, "n_gpus": world,
            "sessions": sessions, "chunks": chunks, "rewinds_per_session": n_rewinds, "every": every,
            "served_fps": tot["frames"] / tmax, "time_s": tmax, **tot,
            "save_gbs": min(r["save_gbs"] for r in allres), "load_gbs": min(r["load_gbs"] for r in allres),
            "peer_restore_gbs": min((r["peer_restore_gbs"] for r in allres if r["peer_restore_gbs"]), default=None),
            "state_bytes": allres[0]["state_bytes"], "note": "GB/s counts read + write bytes"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--chunks", type=int, default=16)
    ap.add_argument("--rewinds", type=int, default=6)
    ap.add_argument("--every", type=int, default=2)
    ap.add_argument("--migrations", type=int, default=2, help="cross-GPU restores per rank")
    ap.add_argument("--max-checkpoints", type=int, default=None, help="checkpoints held per rank (LRU)")
    ap.add_argument("--config", default="mg2")
    a = ap.parse_args()
    rank, world, local = (int(os.environ.get(k, d)) for k, d in (("RANK", 0), ("WORLD_SIZE", 1), ("LOCAL_RANK", 0)))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    from .config import PRESETS
    from .static import B200StaticMG
    cfg = PRESETS[a.config]
    S = B200StaticMG(cfg, device=f"cuda:{local}", seed=0)
    S.add_image("img0", seed=7, max_chunks=a.chunks + 2)
    S.capture(warmup=1)
    res = run(S, rank, world, a.sessions, a.chunks, a.rewinds, a.every, a.migrations, a.max_checkpoints)
    allres = [res]
    if world > 1:
        allres = [None] * world
        torch.distributed.all_gather_object(allres, res)
    if rank == 0:
        print(json.dumps(summarize(allres, world, a.sessions, a.chunks, a.rewinds, a.every, cfg.name)), flush=True)
    S.graphs = {}
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
