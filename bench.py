"""Benchmark: MG2-shaped DiT chunk (config[1]) on B200, one independent session per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one steady-state chunk (4 denoising forwards at t = 1000/750/500/250 with the
flow-matching update, then the context forward at t = 0 that rewrites the 30 history
buffers) of the 30-block Matrix-Game-2-shaped DiT with 15 action blocks, seeded synthetic
weights and inputs.  Metric: frames per second (12 pixel frames per chunk), whole job.

* ``value``: K replays of the captured steady-chunk CUDA graph back to back, inputs resident
  in HBM, CUDA events on the launching stream; every chunk streams 3.2 GB of weights, far
  more than the 126 MB L2, so no flush is needed between steps.
* ``e2e``: K calls of the public API ``B200StaticMG.gen_chunk(path, k)`` (host prep, H2D of the
  chunk's action windows and chunk index from pinned memory, graph replay, output clone) plus a
  D2H read of each chunk's latent into pinned memory, timed with CUDA events.
* ``roofline``: the dominant kernel (the tcgen05 GEMM; FFN-up shape [2640 x 1536] x [8960 x 1536])
  timed alone with CUDA events; algorithmic flops 2 M N K per launch against the measured bf16
  burst peak.
* ``cpu_baseline`` / ``--impl reference``: the reference forward restated on the CPU (the oracle
  port; the reference's own GPU path needs the un-vendored official package), all host threads,
  on a bounded sample: one full forward of a 2-block MG2-width slice (one action block),
  scaled by 15 slices x 5 forwards per chunk.

Multi-GPU (torchrun): every rank runs its own session; there is no collective on the data path
(sessions are independent).  Timing is bracketed by a barrier and synchronize; the job time is
the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from fastworld_b200.config import chunk_flops  # noqa: E402

METRIC = "MG2-shape DiT chunk ms & FPS at 1 GPU; session FPS at 1/2/4/8 B200"
FRAMES_PER_CHUNK = 12


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 4 + i and r[4 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": float(self.rows[0][2]),
                "reasons": reasons, "samples": len(self.rows)}


def cpu_sample_seconds(threads=None):
    """Time one forward of a 2-block MG2-width slice (block 1 with the action module) with the
    CPU oracle; returns (seconds per chunk extrapolated, sample seconds, threads)."""
    from fastworld_b200.config import MG2
    from fastworld_b200.prep import action_windows, synthetic_image
    from fastworld_b200.weights import synthetic_state_dict
    from oracle.mg2_oracle import Oracle
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    cfg = MG2.replace(name="mg2_slice", layers=2, action_blocks=(1,))
    orc = Oracle(cfg, synthetic_state_dict(cfg, 0))
    img = synthetic_image(cfg, 1, 4)
    path = [("img0", ("w", "u"))] * 3
    kc, gm = action_windows(cfg, path, 1)
    inputs = {"cc": img["cond_concat"][0, :, 3:6].float(), "vis": img["visual_context"][0].float(), "gm": gm,
              "kc": kc, "k": 1}
    st = orc.new_state()
    x = torch.randn(16, 3, 44, 80)
    t0 = time.time()
    with torch.no_grad():
        orc.net(st, x, 750.0, False, False, inputs)
    dt = time.time() - t0
    return dt * (MG2.layers // 2) * MG2.n_fwd, dt, threads


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from fastworld_b200.config import MG2
    times = []
    for i in range(args.warmup + args.steps):
        chunk_s, sample_s, threads = cpu_sample_seconds()
        if i >= args.warmup:
            times.append(chunk_s)
    chunk_s = sum(times) / len(times)
    fps = FRAMES_PER_CHUNK / chunk_s
    sample = ("one forward of a 2-block MG2-width slice (1 action block) on the CPU oracle port, "
              "x15 slices x5 forwards per chunk")
    line = {"metric": METRIC, "value": fps, "unit": "frames/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": chunk_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "mg2_steady_chunk", "model": MG2.name, "layers": MG2.layers,
                       "tokens": MG2.tokens, "steps": list(MG2.steps) + [0.0]},
            "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def steady_chunk_ms(cfg, args, rank, world, local):
    """Build a session, run chunk 0, capture, warm up, and time steady-chunk graph replays."""
    from fastworld_b200.static import B200StaticMG
    S = B200StaticMG(cfg, device=f"cuda:{local}", seed=0)
    S.add_image("img0", seed=11 + rank, max_chunks=2)
    path = [("img0", ("w", "u")), ("img0", ("a", "l"))]
    S._prep(path, 0)
    S._chunk(True)
    S.capture(warmup=1)
    S._prep(path, 1)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        S.graphs[(False, "gen")].replay()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        S.graphs[(False, "gen")].replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t)
    S.graphs = {}
    del S
    torch.cuda.empty_cache()
    return ms


def run_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    from fastworld_b200 import _lib, ops
    from fastworld_b200.config import MG2, MG2_FP8
    from fastworld_b200.static import B200StaticMG
    cfg = MG2
    S = B200StaticMG(cfg, device=f"cuda:{local}", seed=0)
    S.add_image("img0", seed=11 + rank, max_chunks=2)
    acts = [("w", "u"), ("a", "l"), ("q", "i"), ("d", "j"), ("s", "k"), ("w", "l")]
    n = args.warmup + args.steps + 4

    def path_upto(k):
        return [("img0", acts[(j * 7 + rank) % len(acts)]) for j in range(k + 1)]

    # images provide cond for 2 chunks; the bench reuses chunk slot 1 for all later chunks
    def prep(k):
        p = path_upto(k)
        S._prep(p, min(k, 1))
        S.chunk_info.copy_(torch.tensor([k, 3 * k, 0, 0], dtype=torch.int32), non_blocking=True)

    prep(0)
    c0 = _lib.lib().fw_launch_count()
    S._chunk(True)
    launches_per_chunk = _lib.lib().fw_launch_count() - c0
    torch.cuda.synchronize()
    S.capture(warmup=1)
    stream = torch.cuda.current_stream()
    for k in range(1, 1 + args.warmup):
        prep(k)
        S.graphs[(False, "gen")].replay()
    torch.cuda.synchronize()
    status = S.device_status()
    # ---- value: steady-chunk graph replays, inputs resident
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            S.graphs[(False, "gen")].replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t)
    # ---- e2e: public API gen_chunk + D2H of each latent
    host = torch.empty(S.out.shape, dtype=torch.bfloat16, pin_memory=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for k in range(1 + args.warmup, 1 + args.warmup + args.steps):
        lat = S.gen_chunk(path_upto(k), 1)
        host.copy_(lat, non_blocking=True)
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = a0.elapsed_time(a1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t)
    status = max(status + S.device_status())
    # ---- roofline of the dominant kernel (tcgen05 GEMM, FFN-up shape), timed alone
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(cfg.tokens, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(cfg.ffn, cfg.dim, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(cfg.ffn, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        ops.gemm(A, B, bias, "gelu_tanh")
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    r0.record(stream)
    for _ in range(reps):
        ops.gemm(A, B, bias, "gelu_tanh")
    r1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = r0.elapsed_time(r1) / reps
    peak_tf, _, peak_kind = peaks()
    gflop = 2.0 * cfg.tokens * cfg.ffn * cfg.dim / 1e9
    achieved = gflop / gemm_ms  # TFLOP/s (GF per ms)
    traffic = None
    prof = os.path.join(ROOT, "profiles", "gemm_ffn_up_mg2.json")
    if os.path.exists(prof):
        traffic = json.load(open(prof)).get("dram_bytes_per_launch")
    flops_all, flops_main = chunk_flops(cfg)
    h2d = S.gm.numel() * 2 + S.kc.numel() * 2 + 16
    d2h = S.out.numel() * 2
    variants = {}
    if not args.no_fp8:   # same chunk with e4m3 block linears
        S.graphs = {}
        S = None
        torch.cuda.empty_cache()
        ms8 = steady_chunk_ms(MG2_FP8, args, rank, world, local)
        variants["fp8"] = {"ms_per_step": ms8, "value": world * FRAMES_PER_CHUNK / (ms8 / 1e3), "unit": "frames/s",
                           "speedup_vs_bf16": ms / ms8, "linear": "e4m3, per-channel weight / per-token scales"}
    line = None
    if rank == 0:
        fps = world * FRAMES_PER_CHUNK / (ms / 1e3)
        e2e_fps = world * FRAMES_PER_CHUNK / (e2e_ms / 1e3)
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu_chunk_s, sample_s, threads = cpu_sample_seconds()
            cpu = {"value": FRAMES_PER_CHUNK / cpu_chunk_s, "unit": "frames/s", "cores": threads, "kind": "port",
                   "sample": f"one forward of a 2-block MG2-width slice (1 action block), {sample_s:.1f} s, "
                             "x15 slices x5 forwards per chunk"}
        line = {"metric": METRIC, "value": fps, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "mg2_steady_chunk", "model": "MG2-shaped causal Wan DiT, 30 blocks, "
                           "15 action blocks, 12x128 heads, ffn 8960", "tokens": cfg.tokens, "history": cfg.tokens,
                           "steps": list(cfg.steps) + [0.0], "sessions_per_gpu": 1,
                           "parallelism": f"sessions x{world}", "l2": "inputs larger than L2 (3.2 GB of weights "
                           "per forward)", "chunk_tflop": flops_all / 1e12,
                           "chunk_tflops_achieved": flops_all / 1e12 / (ms / 1e3)},
                "e2e": {"value": e2e_fps, "unit": "frames/s", "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h},
                "gpu_launches": launches_per_chunk * args.steps,
                "roofline": {"bound": "tensor", "kernel": "gemm_bf16_kernel<256> (FFN-up 2640x8960x1536, GELU)",
                             "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                             "peak_kind": f"{peak_kind} bf16 burst", "traffic": traffic,
                             "launch_ms": gemm_ms, "algorithmic_gflop": gflop},
                "cpu_baseline": cpu, "clocks": clk.summary(), "device_status": status, "variants": variants}
        print(json.dumps(line), flush=True)
    if S is not None:
        S.graphs = {}
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-fp8", action="store_true", help="skip the e4m3 variant (configs[2])")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
