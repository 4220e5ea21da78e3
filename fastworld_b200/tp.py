"""the Wan-14B-shaped causal DiT, tensor-parallel over 1/2/4/8 GPUs.

    python -m fastworld_b200.tp [--config wan14b] [--chunks 3] [--warmup 1] [--graph]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m fastworld_b200.tp

One session whose heads and FFN columns are split over the N ranks (``B200StaticMG(...,
tp_group=True)``); every chunk runs 4 denoising forwards and the context forward, each block
all-reducing (NCCL, on the launch stream) the row-parallel outputs of sa.o, ca.o and ffn.2
and the per-token sums of squares of the q/k RMSNorms.  Chunks 0 and 1 fill the 2-chunk
history window; the timed chunks are steady (keys = 2 history chunks + the current one).

Reports (rank 0, one JSON line): steady chunk latency (CUDA events, max over ranks), frames per
second (12 pixel frames per chunk), algorithmic TFLOP/s per GPU and as a fraction of the
measured bf16 peak, and the time of one standalone NCCL all-reduce of a [tokens, dim] bf16 partial
(the collective of a row-parallel linear) for comparison.  ``--nccl`` runs the engine's
collectives on NCCL instead of its own peer-memory kernels.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch


def _time_calls(fn, reps: int = 10, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def measure(cfg, rank: int, world: int, local: int, chunks: int = 3, warmup: int = 1, graph: bool = True,
            nccl: bool = False, group=None):
    """Build the tensor-parallel session over the default process group (collective: every
    rank calls this with the same arguments), play chunks 0 and 1 (history fill) and ``warmup``
    steady chunks, then time ``chunks`` steady chunks; afterwards time one all-reduce of a
    row-parallel partial and one row-parallel reduction step alone.  Returns this rank's times."""
    from . import _lib
    from .static import B200StaticMG
    dev = torch.device(f"cuda:{local}")
    S = B200StaticMG(cfg, device=dev, seed=0, tp_group=True if world > 1 else None, tp_peers=not nccl)
    n = 2 + warmup + chunks
    S.add_image("img0", seed=7, max_chunks=n + 1)
    path = [("img0", ("w", "u"))] * (n + 1)
    if graph:
        S.capture(warmup=1)
    for k in range(2 + warmup):
        S.gen_chunk(path, k, graph=graph)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier(group=group)
    ms = []
    for k in range(2 + warmup, n):
        S._prep(path, k)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph:
            S.graphs[(False, "gen")].replay()
        else:
            S._chunk(False)
        e1.record()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    status = S.device_status()
    ar_ms = rp_ms = None
    if world > 1:
        L = _lib.lib()
        st = _lib.stream_ptr(torch.cuda.current_stream())
        buf = torch.zeros(cfg.tokens, cfg.dim, dtype=torch.bfloat16, device=dev)
        # one all-reduce of a row-parallel partial on the engine's communicator
        ar_ms = _time_calls(lambda: _lib.check(L.fw_tp_allreduce(S._h, buf.data_ptr(), buf.numel(), _lib.DT_BF16,
                                                                 st), "fw_tp_allreduce"))
        # one row-parallel reduction step exactly as the engine runs it (sum + bias + residual)
        rp_ms = _time_calls(lambda: _lib.check(L.fw_tp_reduce_once(S._h, st), "fw_tp_reduce_once"))
        status = [max(a, b) for a, b in zip(status, S.device_status())]
        del buf
    S.graphs = {}
    del S
    torch.cuda.empty_cache()
    return {"ms": ms, "status": status, "ar_ms": ar_ms, "rp_ms": rp_ms}


def summarize(allres, cfg, world: int, graph: bool, nccl: bool, chunks: int) -> dict:
    from .config import chunk_flops
    chunk_ms = max(max(r["ms"]) for r in allres)
    med = sorted(max(r["ms"][i] for r in allres) for i in range(chunks))[chunks // 2]
    flops, _ = chunk_flops(cfg)
    peak = json.load(open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                       "MEASURED_PEAKS.json")))["bf16_tflops"]
    per_gpu = flops / world / 1e12 / (med / 1e3)
    ar = allres[0]["ar_ms"]
    return {"workload": "wan14b tensor-parallel chunk (BASELINE configs[4])", "config": cfg.name, "tp": world,
            "tokens": cfg.tokens, "history_tokens": cfg.hist_chunks * cfg.tokens, "graph": graph,
            "collectives": ("nccl" if nccl else "peer-memory kernels") if world > 1 else None,
            "chunk_ms_median": med, "chunk_ms_max": chunk_ms, "fps": 12 / (med / 1e3),
            "chunk_tflop": flops / 1e12, "tflops_per_gpu": per_gpu, "frac_of_measured_bf16_peak": per_gpu / peak,
            "allreduce_ms": ar, "row_parallel_step_ms": max(r["rp_ms"] for r in allres) if ar else None,
            "row_parallel_steps_per_chunk": 3 * cfg.layers * cfg.n_fwd if world > 1 else 0,
            "allreduce_busbw_gbs": (2 * (world - 1) / world * cfg.tokens * cfg.dim * 2 / (ar / 1e3) / 1e9)
            if ar else None,
            "status_ok": all(r["status"][0] == 0 for r in allres)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="wan14b")
    ap.add_argument("--chunks", type=int, default=3, help="timed steady chunks")
    ap.add_argument("--warmup", type=int, default=1, help="untimed steady chunks after chunks 0 and 1")
    ap.add_argument("--graph", action="store_true", help="replay captured CUDA graphs instead of eager launches")
    ap.add_argument("--nccl", action="store_true", help="NCCL collectives instead of the peer-memory kernels")
    a = ap.parse_args()
    rank, world, local = (int(os.environ.get(k, d)) for k, d in (("RANK", 0), ("WORLD_SIZE", 1), ("LOCAL_RANK", 0)))
    torch.cuda.set_device(local)
    if world > 1:
        torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    from .config import PRESETS
    cfg = PRESETS[a.config]
    res = measure(cfg, rank, world, local, a.chunks, a.warmup, a.graph, a.nccl)
    allres = [res]
    if world > 1:
        allres = [None] * world
        torch.distributed.all_gather_object(allres, res)
    if rank == 0:
        print(json.dumps(summarize(allres, cfg, world, a.graph, a.nccl, a.chunks)), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
