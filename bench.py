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
* ``cpu_baseline`` (N = 1): the reference forward restated on the CPU (the oracle port; the
  reference's own GPU path needs the un-vendored official package), all host threads: the
  chunk prologue and one complete 30-block steady forward are timed, chunk = prologue + 5
  forwards.  ``--impl reference``: each step is one complete 30-block forward of a steady chunk
  on the oracle port, cycling through the chunk's 5 forwards (prologue in the first), so every 5
  steps are one complete chunk; warm-up steps are one block forward each.
* ``variants``: ``fp8`` (configs[2], every N); ``tp14b`` (configs[4]: a steady Wan-14B-shaped chunk
  tensor-parallel over the N ranks, every N); for N > 1 also ``explore`` (configs[3]: 64 sessions
  from one image, prefix-cache branching, cross-GPU checkpoint restores over NVLink) and
  ``tp_parity`` (a tensor-parallel test model over the N ranks: ranks bit-identical, latents
  against the CPU oracle); ``taehv`` (every N: the TAEHV decoder on one chunk's latent, ms per
  chunk, TFLOP/s, and the served frame rate of DiT chunk + decoder); ``lingbot`` (N = 1: the
  LingBot-World-v2 runtime's steady chunk at its own shape).

Multi-GPU (torchrun): every rank runs its own session; there is no collective on the data path
of ``value`` (sessions are independent).  Timing is bracketed by a barrier and synchronize; the
job time is the max over ranks.
"""
from __future__ import annotations

import argparse
import datetime
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


class CpuChunk:
    """The steady chunk of configs[1] on the CPU oracle port, one forward per call of ``step``:
    calls 0-3 are the denoising forwards (flow-matching update between them), call 4 the
    context forward that rewrites the history; call 0 also runs the chunk prologue (context MLP
    and every layer's cross-attention K/V).  History and action state start as N(0, 1)."""

    def __init__(self, threads=None, cfg=None):
        from fastworld_b200.config import MG2
        from fastworld_b200.prep import action_windows, synthetic_image
        from fastworld_b200.weights import synthetic_state_dict
        from oracle.mg2_oracle import Oracle
        self.threads = threads or os.cpu_count()
        torch.set_num_threads(self.threads)
        self.cfg = cfg = cfg or MG2
        self.orc = Oracle(cfg, synthetic_state_dict(cfg, 0))
        g = torch.Generator().manual_seed(3)
        self.st = st = self.orc.new_state()
        for nm in ("hk", "hv"):
            st[nm].copy_(torch.randn(st[nm].shape, generator=g).bfloat16().float())
        for nm in ("mk", "mv", "kk", "kv"):
            for i in st[nm]:
                st[nm][i] = torch.randn(st[nm][i].shape, generator=g).bfloat16().float()
        img = synthetic_image(cfg, 1, 2)
        path = [("img0", ("w", "u")), ("img0", ("a", "l"))]
        kc, gm = action_windows(cfg, path, 1)
        self.inputs = {"cc": img["cond_concat"][0, :, 3:6].float(), "vis": img["visual_context"][0].float(),
                       "gm": gm, "kc": kc, "k": 1}
        self.x_in = torch.randn(cfg.lat_ch, cfg.frames, cfg.lat_h, cfg.lat_w, generator=g).bfloat16().float()
        self.noise = [torch.randn(cfg.frames, cfg.lat_ch, cfg.lat_h, cfg.lat_w, generator=g).bfloat16().float()
                      for _ in cfg.steps[1:]]
        self.j, self.x, self.den, self.ctx = 0, None, None, None

    def prologue(self):
        o = self.orc
        ctx = o.context(self.inputs["vis"])
        self.ctx = [o.cross_kv(i, ctx) for i in range(self.cfg.layers)]
        self.x = self.x_in

    @torch.no_grad()
    def step(self):
        from oracle.mg2_oracle import sigma_of
        o, c, j = self.orc, self.cfg, self.j
        if j == 0:
            self.prologue()
        n = len(c.steps)
        if j < n:
            self.den = o.net(self.st, self.x, c.steps[j], False, False, self.inputs, self.ctx)
            if j < n - 1:
                sg = sigma_of(c.steps[j + 1])
                self.x = o.i((1 - sg) * self.den + sg * self.noise[j].transpose(0, 1))
        else:
            o.net(self.st, self.den, 0.0, False, True, self.inputs, self.ctx)
        self.j = (j + 1) % (n + 1)

    @torch.no_grad()
    def warm(self):
        """One block forward (the CPU path has only its allocator and thread pool to warm)."""
        from oracle.mg2_oracle import rope_table
        o, c = self.orc, self.cfg
        if self.ctx is None:
            self.prologue()
        _, e0 = o.time_embed(750.0)
        xs = torch.zeros(c.tokens, c.dim)
        st = {k: (dict(v) if isinstance(v, dict) else v) for k, v in self.st.items()}
        o.block(c.action_blocks[0], xs, e0[None].expand(c.frames, 6, c.dim), rope_table(c, 1, o.freqs), st, False,
                False, self.ctx[c.action_blocks[0]], self.inputs["gm"], self.inputs["kc"], c.frames)


def cpu_chunk_seconds():
    """Our arm's CPU baseline: the chunk prologue and one complete steady forward (t = 750),
    each timed once; a chunk is the prologue + 5 forwards (the five cost the same but for the
    context forward's history write).  Returns (chunk s, forward s, prologue s, threads)."""
    cc = CpuChunk()
    t0 = time.time()
    cc.prologue()
    t_pro = time.time() - t0
    t0 = time.time()
    with torch.no_grad():
        cc.orc.net(cc.st, cc.x, 750.0, False, False, cc.inputs, cc.ctx)
    t_fwd = time.time() - t0
    return t_pro + (len(cc.cfg.steps) + 1) * t_fwd, t_fwd, t_pro, cc.threads


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from fastworld_b200.config import MG2
    cc = CpuChunk()
    for _ in range(args.warmup):
        cc.warm()
    per_chunk = len(MG2.steps) + 1
    times = []
    for _ in range(args.steps):
        t0 = time.time()
        cc.step()
        times.append(time.time() - t0)
    step_s = sum(times) / len(times)
    chunk_s = step_s * per_chunk
    fps = FRAMES_PER_CHUNK / chunk_s
    sample = (f"{args.steps} complete 30-block forwards of steady chunks ({args.steps / per_chunk:g} chunks: "
              f"4 denoising forwards + the context forward each, prologue in the first), measured; "
              f"warm-up steps one block forward each")
    line = {"metric": METRIC, "value": fps, "unit": "frames/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "mg2_steady_chunk", "model": MG2.name, "layers": MG2.layers,
                       "tokens": MG2.tokens, "steps": list(MG2.steps) + [0.0],
                       "step": "one complete 30-block forward; 5 steps = one steady chunk",
                       "chunk_ms": chunk_s * 1e3, "forward_ms": [t * 1e3 for t in times]},
            "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": cc.threads, "kind": "port", "sample": sample},
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
    t_start = time.time()
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    from fastworld_b200 import _lib, ops
    from fastworld_b200.config import MG2, MG2_FP8, MG2_FP8_FFN
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
    ctl = torch.distributed.new_group(backend="gloo", timeout=datetime.timedelta(seconds=600)) if world > 1 else None
    if world > 1 and not args.no_explore and agree(time.time() - t_start < args.variant_budget, world, ctl):
        variants["explore"] = guarded(lambda: explore_variant(S, rank, world, ctl), world, ctl)
    S.graphs = {}
    S = None
    torch.cuda.empty_cache()
    if not args.no_fp8 and agree(time.time() - t_start < args.variant_budget, world, ctl):
        # same chunk with e4m3 block linears
        def fp8(cfg8, what):
            ms8 = steady_chunk_ms(cfg8, args, rank, world, local)
            return {"ms_per_step": ms8, "value": world * FRAMES_PER_CHUNK / (ms8 / 1e3), "unit": "frames/s",
                    "speedup_vs_bf16": ms / ms8, "linear": what}
        variants["fp8"] = guarded(lambda: fp8(MG2_FP8, "every block linear e4m3, per-channel weight / per-token "
                                              "activation scales"), world, ctl)
        variants["fp8_ffn"] = guarded(lambda: fp8(MG2_FP8_FFN, "FFN linears (ffn.0, ffn.2) e4m3, the rest bf16"),
                                      world, ctl)
    if not args.no_tp and agree(time.time() - t_start < args.variant_budget, world, ctl):
        variants["tp14b"] = guarded(lambda: tp14b_variant(rank, world, local, ctl), world, ctl)
    if world > 1 and not args.no_tp and agree(time.time() - t_start < args.variant_budget, world, ctl):
        variants["tp_parity"] = guarded(lambda: tp_parity_variant(rank, world, local, ctl), world, ctl)
    if not args.no_taehv and agree(time.time() - t_start < args.variant_budget, world, ctl):
        variants["taehv"] = guarded(lambda: taehv_variant(ms, rank, world, ctl), world, ctl)
    if world == 1 and not args.no_lingbot and time.time() - t_start < args.variant_budget:
        variants["lingbot"] = guarded(lambda: lingbot_variant(rank, world, ctl), world, ctl)
    line = None
    if rank == 0:
        fps = world * FRAMES_PER_CHUNK / (ms / 1e3)
        e2e_fps = world * FRAMES_PER_CHUNK / (e2e_ms / 1e3)
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu_chunk_s, fwd_s, pro_s, threads = cpu_chunk_seconds()
            cpu = {"value": FRAMES_PER_CHUNK / cpu_chunk_s, "unit": "frames/s", "cores": threads, "kind": "port",
                   "sample": f"the chunk prologue ({pro_s:.1f} s) and one complete 30-block steady forward "
                             f"({fwd_s:.1f} s), measured; chunk = prologue + 5 forwards"}
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
    if world > 1:
        torch.distributed.barrier(group=ctl)
        torch.distributed.destroy_process_group()


def agree(flag: bool, world: int, ctl) -> bool:
    """True when every rank passes True (the ranks must take the same collective steps)."""
    if world == 1:
        return bool(flag)
    got = [None] * world
    torch.distributed.all_gather_object(got, bool(flag), group=ctl)
    return all(got)


def guarded(fn, world: int, ctl):
    """Run a variant on every rank; rank 0 gets its result, or the first error any rank hit."""
    try:
        res, err = fn(), None
    except Exception as e:   # a variant's failure must not lose the main line
        res, err = None, f"{type(e).__name__}: {e}"[:400]
    if world > 1:
        errs = [None] * world
        torch.distributed.all_gather_object(errs, err, group=ctl)
        err = next((e for e in errs if e), None)
    return {"error": err} if err else res


def explore_variant(S, rank, world, ctl):
    """configs[3] over the N ranks on this rank's captured session (64 sessions x 16 chunks,
    6 rewinds each, a checkpoint every 2 chunks, at most 48 held per GPU, cross-GPU restores)."""
    from fastworld_b200 import explore
    S.add_image("explore", seed=7, max_chunks=18)
    res = explore.run(S, rank, world, sessions=64, chunks=16, n_rewinds=6, every=2, migrations=2,
                      max_checkpoints=48, group=ctl, img="explore")
    allres = [None] * world
    torch.distributed.all_gather_object(allres, res, group=ctl)
    return explore.summarize(allres, world, 64, 16, 6, 2, "mg2") if rank == 0 else None


def taehv_variant(chunk_ms, rank, world, ctl):
    """The decoder after the DiT (the reference's TinyVAE, TAEHV taew2_1): every rank decodes its
    own session's chunks; decode time is the max over ranks."""
    from fastworld_b200.vae import TAEW2_1
    dms, vae = taehv_decode_ms(10)
    del vae
    torch.cuda.empty_cache()
    if world > 1:
        got = [None] * world
        torch.distributed.all_gather_object(got, dms, group=ctl)
        dms = max(got)
    peak_tf, _, peak_kind = peaks()
    tf = TAEW2_1.flops() / 1e12 / (dms / 1e3)
    fr = TAEW2_1.frames_out
    return {"workload": "TinyVAE (TAEHV taew2_1) streaming decode of one MG2 latent chunk: [1, 16, 3, 44, 80] -> "
                        "12 frames of 352 x 640 (fp16 activations, fp32 accumulate; one library-held graph)",
            "ms_per_chunk": dms, "frames_per_s": world * fr / (dms / 1e3), "algorithmic_gflop": TAEW2_1.flops() / 1e9,
            "tflops": tf, "frac_of_peak": tf / peak_tf, "peak_kind": f"{peak_kind} bf16 burst",
            "dit_plus_decoder_fps": world * fr / ((chunk_ms + dms) / 1e3),
            "reference_ms_per_chunk_published": 10.4}


def lingbot_variant(rank, world, ctl):
    """The LingBot-World-v2 runtime at its shape (Wan-1.3B, 4 latent frames = 6032 tokens per
    chunk, an 18-frame window = 27144 keys with a 6-frame sink): steady chunks (plan (14, 18),
    roll [10:18] -> [6:14]) replayed from the captured graph; every rank runs its own session."""
    from fastworld_b200.lingbot import LINGBOT, B200StaticLingbot, synthetic_inputs
    cfg = LINGBOT
    I = synthetic_inputs(cfg, 9, seed=0, text_tokens=120)
    S = B200StaticLingbot(cfg, device=f"cuda:{torch.cuda.current_device()}", seed=0)
    S.set_session(I)
    S.capture()
    for k in range(5):                     # chunks 0-4: fill the window, reach the steady plan
        S.gen_chunk(k)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for k in range(5, 9):
        S._prep(k)
        e0.record()
        S.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    status = S.device_status()
    del S
    torch.cuda.empty_cache()
    ms = sorted(times)[len(times) // 2]
    if world > 1:
        got = [None] * world
        torch.distributed.all_gather_object(got, ms, group=ctl)
        ms = max(got)
    fl = cfg.flops()
    peak_tf, _, peak_kind = peaks()
    return {"workload": "LingBot-World-v2 causal chunk (Wan-1.3B I2V + camera injector + text cross-attention), "
                        "6032 tokens over a 27144-key window with a 6-frame sink, 4 steps + the key refresh",
            "ms_per_chunk": ms, "frames_per_s": world * 4 * cfg.chunk / (ms / 1e3),
            "chunk_tflop": fl["total"] / 1e12, "tflops": fl["total"] / 1e12 / (ms / 1e3),
            "frac_of_peak": fl["total"] / 1e12 / (ms / 1e3) / peak_tf, "peak_kind": f"{peak_kind} bf16 burst",
            "attention_share_of_flops": fl["attention"] / fl["total"], "graphs": 1, "status_ok": status == 0,
            "reference_ms_per_chunk_published_h100": 843}


def tp14b_variant(rank, world, local, ctl):
    """one Wan-14B-shaped session tensor-parallel over the N ranks (peer-memory
    reductions), steady chunks replayed from captured graphs."""
    from fastworld_b200 import tp
    from fastworld_b200.config import WAN14B
    res = tp.measure(WAN14B, rank, world, local, chunks=3, warmup=1, graph=True, nccl=False, group=ctl)
    allres = [res]
    if world > 1:
        allres = [None] * world
        torch.distributed.all_gather_object(allres, res, group=ctl)
    if rank != 0:
        return None
    out = tp.summarize(allres, WAN14B, world, True, False, 3)
    if out["row_parallel_step_ms"]:
        out["row_parallel_share_of_chunk"] = (out["row_parallel_step_ms"] * out["row_parallel_steps_per_chunk"] /
                                              out["chunk_ms_median"])
    return out


TP_PARITY_PATH = [("img0", ("w", "u")), ("img0", ("a", "l")), ("img0", ("q", "i")), ("img0", ("d", "j"))]


def tp_parity_variant(rank, world, local, ctl):
    """A tensor-parallel test model (8 heads, FFN 2048, 2 blocks, 2-chunk history) over the N
    ranks, chunks 0-3: every rank's latent must be bit-identical; rank 0 checks the latents
    and every rank's history heads against the CPU oracle (rel-L2)."""
    from fastworld_b200.config import SMALL_TP
    from fastworld_b200.prep import action_windows, synthetic_image
    from fastworld_b200.static import B200StaticMG
    from fastworld_b200.weights import synthetic_state_dict
    cfg = SMALL_TP.replace(name="small_tp8", heads=8, dim=1024, ffn=2048)
    sd = synthetic_state_dict(cfg, 0)
    img = synthetic_image(cfg, 5, 5)
    S = B200StaticMG(cfg, sd, device=f"cuda:{local}", tp_group=True)
    S.add_image("img0", img)
    outs, inputs = [], []
    for k in range(4):
        S._prep(TP_PARITY_PATH, k)
        inputs.append((S.x_in.cpu(), [n.cpu() for n in S.noise]))
        S._chunk(k == 0)
        outs.append(S.out.cpu())
    torch.cuda.synchronize()
    res = {"outs": outs, "hk": [h.cpu() for h in S.hk], "status": S.device_status()}
    del S
    allres = [None] * world
    torch.distributed.all_gather_object(allres, res, group=ctl)
    if rank != 0:
        return None
    from oracle.mg2_oracle import Oracle
    same = all(torch.equal(allres[0]["outs"][k], r["outs"][k]) for r in allres for k in range(4))
    orc = Oracle(cfg, sd)
    st = orc.new_state()
    rel = lambda a, b: float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))  # noqa: E731
    e_out = []
    with torch.no_grad():
        for k in range(4):
            s = cfg.frames * k
            kc, gm = action_windows(cfg, TP_PARITY_PATH, k)
            inp = {"cc": img["cond_concat"][0, :, s:s + cfg.frames].float(), "vis": img["visual_context"][0].float(),
                   "gm": gm, "kc": kc, "k": k}
            x_in, noise = inputs[k]
            ref = orc.chunk(st, x_in[0].float(), [n.float() for n in noise], inp, k == 0)
            e_out.append(rel(outs[k][0], ref))
    hl = cfg.heads // world
    e_hist = max(rel(allres[r]["hk"][i][0], st["hk"][i][:, r * hl:(r + 1) * hl]) for r in range(world)
                 for i in range(cfg.layers))
    return {"config": f"{cfg.name}: dim {cfg.dim}, {cfg.heads} heads, ffn {cfg.ffn}, {cfg.layers} blocks, "
                      f"{cfg.hist_chunks}-chunk history", "tp": world, "chunks": 4, "ranks_identical": same,
            "oracle_rel_l2": e_out, "history_rel_l2_max": e_hist, "bound": 1.2e-2,
            "pass": same and max(e_out) < 1.2e-2 and e_hist < 1.2e-2,
            "status_ok": all(r["status"][0] == 0 for r in allres)}


# ---------------------------------------------------------------- single-kernel workloads
# Small, self-terminating runs of one kernel for ncu captures and CUDA-event timing:
#   python bench.py --kernel gemm|gemm_resid|attn|ln|ln14|rms|copy|fp8_peak [--reps 3]
#   python bench.py --kernel chunk [--chunks 2] [--config mg2|mg2_fp8]   (eager chunks)

def chunk(n: int, config: str = "mg2") -> None:
    from fastworld_b200 import _lib
    from fastworld_b200.config import PRESETS
    from fastworld_b200.static import B200StaticMG
    S = B200StaticMG(PRESETS[config], seed=0)
    S.add_image("img0", seed=3, max_chunks=n + 1)
    path = [("img0", ("w", "u"))] * (n + 1)
    for k in range(n):
        S._prep(path, k)
        c0 = _lib.lib().fw_launch_count()
        S._chunk(k == 0)
        torch.cuda.synchronize()
        print(f"chunk {k}: {_lib.lib().fw_launch_count() - c0} launches, status {S.device_status()}")


def gemm(reps: int) -> None:
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(2640, 1536, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(8960, 1536, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(8960, device="cuda", dtype=torch.bfloat16)
    for _ in range(reps):
        ops.gemm(A, B, bias, "gelu_tanh")
    torch.cuda.synchronize()
    print("gemm ok")


def gemm_resid(reps: int) -> None:
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(2640, 1536, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(1536, 1536, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(1536, device="cuda", dtype=torch.bfloat16)
    resid = torch.zeros(2640, 1536, device="cuda")
    gate = torch.ones(3, 1536, device="cuda")
    for _ in range(reps):
        ops.gemm_resid_(resid, A, B, bias, gate, 880)
    torch.cuda.synchronize()
    print("gemm_resid ok")


def attn(reps: int) -> None:
    """Steady self-attention (12 heads, 2640 queries over 2640 history + 2640 current keys) and
    cross-attention (2640 queries over 257 context keys), MG2 shape, and the LingBot window
    (6032 queries over 27144 keys); timed through recorded graphs of back-to-back launches."""
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    r = lambda n: torch.randn(n, 12, 128, device="cuda", generator=g).to(torch.bfloat16)  # noqa: E731
    q, k0, v0, k1, v1 = r(2640), r(2640), r(2640), r(2640), r(2640)
    kc, vc = r(257), r(257)
    meta = torch.tensor([2640, 2640], dtype=torch.int32, device="cuda")
    meta_x = torch.tensor([257, 0], dtype=torch.int32, device="cuda")
    for _ in range(reps):
        ops.attention(q, k0, v0, k1, v1, meta)
    torch.cuda.synchronize()
    ms = _graph_ms([lambda: ops.attention(q, k0, v0, k1, v1, meta)] * 4)
    msx = _graph_ms([lambda: ops.attention(q, kc, vc, kc, vc, meta_x)] * 4)
    fl, flx = 4.0 * 2640 * 5280 * 128 * 12, 4.0 * 2640 * 257 * 128 * 12
    print(f"attention self {ms * 1e3:.1f} us ({fl / ms / 1e9:.0f} TFLOP/s), cross {msx * 1e3:.1f} us "
          f"({flx / msx / 1e9:.0f} TFLOP/s)")
    # the LingBot window: 6032 queries over 27144 keys (one segment), 12 heads
    ql, kl, vl = r(6032), r(27144), r(27144)
    meta_l = torch.tensor([27144, 0], dtype=torch.int32, device="cuda")
    for _ in range(reps):
        ops.attention(ql, kl, vl, kl, vl, meta_l)
    torch.cuda.synchronize()
    msl = _graph_ms([lambda: ops.attention(ql, kl, vl, kl, vl, meta_l)] * 4)
    fll = 4.0 * 6032 * 27144 * 128 * 12
    print(f"attention LingBot window {msl * 1e3:.1f} us ({fll / msl / 1e9:.0f} TFLOP/s)")


def gemm_vs_cublas(reps: int) -> None:
    """The engine's bf16 GEMM (plain bf16 epilogue) against cuBLAS (torch.matmul) on the same
    operands: the MG2, LingBot and 14B linear shapes and 8192^3, both timed through recorded
    graphs of back-to-back launches.  A comparison only: no product path calls cuBLAS."""
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    shapes = [("mg2 qkv", 2640, 4608, 1536), ("mg2 o-proj", 2640, 1536, 1536), ("mg2 ffn.0", 2640, 8960, 1536),
              ("mg2 ffn.2", 2640, 1536, 8960), ("lingbot qkv", 6032, 4608, 1536),
              ("lingbot ffn.0", 6032, 8960, 1536), ("14b qkv", 4680, 15360, 5120), ("14b ffn.0", 4680, 13824, 5120),
              ("14b ffn.2", 4680, 5120, 13824), ("8192^3", 8192, 8192, 8192)]
    for name, M, N, K in shapes:
        a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        bt = b.t()
        for _ in range(max(reps, 3)):
            ops.gemm(a, b)
            torch.matmul(a, bt)
        torch.cuda.synchronize()
        ours = _graph_ms([lambda: ops.gemm(a, b)] * 4)
        lib = _graph_ms([lambda: torch.matmul(a, bt)] * 4)
        fl = 2.0 * M * N * K
        print(f"{name:14s} {M}x{N}x{K}: engine {ours * 1e3:8.1f} us {fl / ours / 1e9:6.0f} TFLOP/s | cuBLAS "
              f"{lib * 1e3:8.1f} us {fl / lib / 1e9:6.0f} TFLOP/s | engine / cuBLAS speed {lib / ours:.3f}")


def fp8_peak(reps: int) -> None:
    from fastworld_b200 import ops
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(n, n, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(n, n, device="cuda", generator=g).to(torch.bfloat16)
    a8, sa = ops.quant_e4m3(a)
    b8, sw = ops.quant_e4m3(b)
    fa, fb = a8.view(torch.float8_e4m3fn), b8.view(torch.float8_e4m3fn)
    one = torch.ones((), device="cuda")

    def best(fn, n_rep=10):
        for _ in range(3):
            fn()
        t = 1e9
        for _ in range(n_rep):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            t = min(t, e0.elapsed_time(e1))
        return t
    flop = 2.0 * n ** 3
    t_lib = best(lambda: torch._scaled_mm(fa, fb.t(), one, one, out_dtype=torch.bfloat16))
    t_ours = best(lambda: ops.gemm_e4m3(a8, sa, b8, sw, None, "none"))
    t_bf16 = best(lambda: torch.matmul(a, b.t()))
    print(f"e4m3 8192^3: library {flop / t_lib / 1e9:.1f} TFLOP/s, fastworld_b200 {flop / t_ours / 1e9:.1f} TFLOP/s; "
          f"bf16 library {flop / t_bf16 / 1e9:.1f} TFLOP/s (burst, best of 10)")




def _events_ms(fn, reps):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _rows(n_sets, make):
    """n_sets independent operand sets (cycled so that back-to-back launches stream from HBM once
    their total exceeds the 126 MB L2)."""
    return [make(i) for i in range(n_sets)]


def _graph_ms(fns, replays=20):
    """Record the launches of ``fns`` (one per operand set) as one library-held graph and time its
    replays with CUDA events: back-to-back launches with no host overhead between them, as inside
    a captured chunk.  Returns ms per launch."""
    from fastworld_b200.graph import LibGraph

    def all_sets():
        for f in fns:
            f()
    all_sets()
    g = LibGraph.record(all_sets)
    for _ in range(3):
        g.replay()
    return _events_ms(g.replay, replays) / len(fns)


def ln(reps: int) -> None:
    """norm1 / norm2 of the MG2 block: LayerNorm of the fp32 residual [2640, 1536] + adaLN
    modulate into bf16; algorithmic bytes 16.2 MB read + 8.1 MB written per launch."""
    from fastworld_b200 import ops
    M, D = 2640, 1536
    g = torch.Generator(device="cuda").manual_seed(0)
    sets = _rows(8, lambda i: (torch.randn(M, D, device="cuda", generator=g),
                               torch.empty(M, D, device="cuda", dtype=torch.bfloat16)))
    shift, scale = torch.randn(D, device="cuda", generator=g) * 0.1, torch.randn(D, device="cuda", generator=g) * 0.1
    fns = [lambda x=x, o=o: ops.layernorm(x, 1e-6, shift=shift, scale=scale, out=o) for x, o in sets]
    for _ in range(reps):
        for f in fns:
            f()
    torch.cuda.synchronize()
    ms = _graph_ms(fns)
    nb = M * D * 6
    print(f"ln_kernel 2640x1536: {ms * 1e3:.2f} us/launch, graph of back-to-back launches over 8 operand sets "
          f"(194 MB > L2): {nb / ms / 1e6:.0f} GB/s")


def ln14(reps: int) -> None:
    """norm1 / norm2 of the Wan-14B block: LayerNorm of the fp32 residual [4680, 5120] + adaLN
    modulate into bf16 (four warps per row); algorithmic bytes 95.8 MB read + 47.9 MB written."""
    from fastworld_b200 import ops
    M, D = 4680, 5120
    g = torch.Generator(device="cuda").manual_seed(0)
    sets = _rows(2, lambda i: (torch.randn(M, D, device="cuda", generator=g),
                               torch.empty(M, D, device="cuda", dtype=torch.bfloat16)))
    shift, scale = torch.randn(D, device="cuda", generator=g) * 0.1, torch.randn(D, device="cuda", generator=g) * 0.1
    fns = [lambda x=x, o=o: ops.layernorm(x, 1e-6, shift=shift, scale=scale, out=o) for x, o in sets]
    for _ in range(reps):
        for f in fns:
            f()
    torch.cuda.synchronize()
    ms = _graph_ms(fns)
    nb = M * D * 6
    print(f"ln_wide_kernel 4680x5120: {ms * 1e3:.2f} us/launch, graph of back-to-back launches over 2 operand sets "
          f"(288 MB > L2): {nb / ms / 1e6:.0f} GB/s")


def rms(reps: int) -> None:
    """q and k RMSNorm + RoPE of the MG2 block ([2640, 1536] bf16 each, in place, as the engine
    runs them); algorithmic bytes 8.1 MB read + 8.1 MB written per tensor + the 1.35 MB RoPE table."""
    from fastworld_b200 import ops
    M, D, hd = 2640, 1536, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    sets = _rows(8, lambda i: torch.randn(M, D, device="cuda", generator=g).bfloat16())
    w = (torch.rand(D, device="cuda", generator=g) + 0.5).bfloat16()
    ang = torch.rand(M, hd // 2, device="cuda", generator=g) * 6.3
    rope = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    fns = [lambda x=x: ops.rms_rope(x, w, rope, hd, out=x) for x in sets]
    for _ in range(reps):
        for f in fns:
            f()
    torch.cuda.synchronize()
    ms = _graph_ms(fns)
    nb = M * D * 4
    print(f"rms_rope8_kernel 2640x1536: {ms * 1e3:.2f} us/launch, graph of back-to-back launches over 8 operand "
          f"sets (130 MB > L2): {nb / ms / 1e6:.0f} GB/s (+ RoPE table)")


def copy(reps: int) -> None:
    """Checkpoint save / restore: one copy of the 649 MB MG2 session state."""
    from fastworld_b200 import ops
    nb = 648990720
    a = torch.empty(nb, dtype=torch.uint8, device="cuda")
    b = torch.empty(nb, dtype=torch.uint8, device="cuda")
    for _ in range(reps):
        ops.copy_(b, a)
    ms = _events_ms(lambda: ops.copy_(b, a), 20)
    print(f"copy_kernel 649 MB: {ms * 1e3:.1f} us, {2 * nb / ms / 1e6:.0f} GB/s (read + write)")


def taehv_decode_ms(replays: int = 10):
    """TinyVAE (taew2_1) on one MG2 latent chunk: warm graph replays timed with CUDA events.
    Returns (ms per chunk, the decoder) after checking the device status."""
    from fastworld_b200.vae import TAEW2_1, TinyVAE
    cfg = TAEW2_1
    vae = TinyVAE("cuda", cfg=cfg, seed=0)
    g = torch.Generator(device="cuda").manual_seed(0)
    lat = torch.randn(1, 16, cfg.lat_frames, cfg.lat_h, cfg.lat_w, device="cuda", generator=g).bfloat16()
    for _ in range(3):
        vae.decode(lat)
    ms = _events_ms(vae.graph.replay, replays)
    if vae.device_status() != 0:
        raise RuntimeError(f"taehv device status {vae.device_status()}")
    return ms, vae


def taehv(reps: int) -> None:
    """The TAEHV decoder on one MG2 latent chunk (12 frames of 352 x 640): graph replays."""
    from fastworld_b200.vae import TAEW2_1
    ms, vae = taehv_decode_ms(max(reps, 3))
    n = vae.graph.num_nodes()
    tf = TAEW2_1.flops() / 1e12 / (ms / 1e3)
    print(f"taehv decode: {ms:.3f} ms per chunk ({n} graph nodes), {TAEW2_1.frames_out / (ms / 1e3):.0f} frames/s, "
          f"{TAEW2_1.flops() / 1e9:.1f} GFLOP algorithmic = {tf:.0f} TFLOP/s")


def lingbot(reps: int) -> None:
    """The LingBot runtime at its shape: steady chunk time from graph replays."""
    out = lingbot_variant(0, 1, None)
    print(json.dumps(out))


def lingbot_chunk(reps: int) -> None:
    """One steady LingBot chunk launched eagerly inside the NVTX range "lb_chunk" (for a launch
    list: ncu --nvtx --nvtx-include "lb_chunk/"), after 6 chunks that reach the steady plan."""
    from fastworld_b200.lingbot import LINGBOT, B200StaticLingbot, synthetic_inputs
    I = synthetic_inputs(LINGBOT, 8, seed=0, text_tokens=120)
    S = B200StaticLingbot(LINGBOT, device="cuda", seed=0)
    S.set_session(I)
    for k in range(6):
        S.gen_chunk(k)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("lb_chunk")
    S.gen_chunk(6, graph=False)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(f"lingbot chunk 6 (eager) done, device status {S.device_status()}")


KERNELS = {"chunk": lambda a: chunk(a.chunks, a.config), "gemm": lambda a: gemm(a.reps), "taehv": lambda a: taehv(a.reps),
           "lingbot": lambda a: lingbot(a.reps), "lingbot_chunk": lambda a: lingbot_chunk(a.reps),
           "gemm_resid": lambda a: gemm_resid(a.reps), "attn": lambda a: attn(a.reps), "ln": lambda a: ln(a.reps),
           "ln14": lambda a: ln14(a.reps), "rms": lambda a: rms(a.reps), "copy": lambda a: copy(a.reps),
           "fp8_peak": lambda a: fp8_peak(a.reps), "gemm_vs_cublas": lambda a: gemm_vs_cublas(a.reps)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--kernel", choices=sorted(KERNELS), help="run one kernel's small workload instead")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--chunks", type=int, default=2)
    ap.add_argument("--config", default="mg2")
    ap.add_argument("--no-fp8", action="store_true", help="skip the e4m3 variant (configs[2])")
    ap.add_argument("--no-tp", action="store_true", help="skip the 14B tensor-parallel variants (configs[4])")
    ap.add_argument("--no-explore", action="store_true", help="skip the explore variant (configs[3], N > 1)")
    ap.add_argument("--no-taehv", action="store_true", help="skip the decoder variant")
    ap.add_argument("--no-lingbot", action="store_true", help="skip the LingBot runtime variant")
    ap.add_argument("--variant-budget", type=float, default=600.0,
                    help="start no further variant once this many seconds have passed")
    args = ap.parse_args()
    if args.kernel:
        KERNELS[args.kernel](args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
