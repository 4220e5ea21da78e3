"""The LingBot-World-v2 causal runtime on the engine's sm_100a kernels: a Wan-1.3B I2V DiT with a
camera injector, text cross-attention and a sink + rolling KV window, served chunk by chunk
(the reference's ``StaticLingbot``, ``fastworld/models/lingbot_v2/static.py:49-320``).

What a chunk computes (``static.py:209-281``): 4 denoising forwards of the DiT over the chunk's
C = 4 latent frames (x0 = x - sigma * flow in fp64, then renoising with the session generator's
noise), then a forward at t = 0 over the denoised latent that refreshes the chunk's keys, and the
end-of-chunk roll of the KV window.  Every forward writes its RoPE'd keys and values into the
per-layer KV buffer at the plan's write offset before attending to the buffer's first
``key_len`` frames; the camera branch (Plücker features -> per-block scale / shift of the
residual) is computed once per chunk (the reference's ``hoist=True``); the prompt's cross-
attention K/V once per prompt.

Plans (``static.py:30-46``): the eager runtime's KV bookkeeping in frames, per chunk
(write offset, key length, roll after the chunk); :func:`eager_plans` restates it and
``tests/test_lingbot_host.py`` pins it against the reference's own function.

The engine keeps the plan of the chunk in device memory, so one captured graph serves every
chunk (the reference records one graph per distinct plan).
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass
from typing import Dict, List, Tuple

import numpy as np
import torch

LOCAL_ATTN, SINK = 18, 6     # frames: KV window and its sink (the reference's LOCAL_ATTN, SINK)


def eager_plans(n: int, C: int, W: int = LOCAL_ATTN, S: int = SINK):
    """Per chunk (roll before it, write offset, key length) in frames, as the eager runtime's
    index bookkeeping produces them (``static.py:30-46``).  roll = (src, dst, frames): frames
    [src, src + n) move to [dst, dst + n)."""
    local_end = global_end = 0
    out = []
    for c in range(n):
        cur_end = (c + 1) * C
        roll = None
        if W != -1 and cur_end > global_end and C + local_end > W:
            ev = C + local_end - W                  # frames evicted past the window
            moved = local_end - ev - S              # non-sink frames that survive
            roll = (S + ev, S, moved)
            local_end = local_end + cur_end - global_end - ev
        else:
            local_end = local_end + cur_end - global_end
        out.append((roll, local_end - C, local_end))
        global_end = cur_end
    return out


def chunk_plans(n: int, C: int, W: int = LOCAL_ATTN, S: int = SINK):
    """Per chunk (write offset, key length, roll after the chunk): the roll the eager runtime
    does at the start of chunk c + 1 is done at the end of chunk c (``static.py:10-13``)."""
    pl = eager_plans(n + 1, C, W, S)
    return [(pl[c][1], pl[c][2], pl[c + 1][0]) for c in range(n)]


def flow_schedule(steps_index=(0, 250, 500, 750), n_train: int = 1000, shift: float = 3.0):
    """Timesteps and the scheduler constants of the 4-step causal-fast loop.

    Shifted flow-matching sigmas s' = shift s / (1 + (shift - 1) s) over s = 1 .. 1/n_train
    (n_train points, then a final 0), timesteps = 1000 s'; the chunk loop uses
    timesteps[steps_index].  Per step i: ``sig_x0[i]`` (fp64) = the sigma whose timestep is
    nearest to t_i (``static.py:110-115``); renoising to t_{i+1} uses alpha = 1 - sigma,
    sigma = the fp32 sigma of t_{i+1} (``static.py:116-125``).  The scheduler itself belongs to
    the un-vendored Wan package: these constants are this build's restatement, shared by the
    engine and the oracle."""
    sigmas32, ts32 = scheduler_tables(n_train, shift)
    t = [float(ts32[i]) for i in steps_index]
    sig_x0 = [float(sigmas32[int(np.argmin(np.abs(ts32.astype(np.float64) - ti)))]) for ti in t]
    an_alpha, an_sigma = [], []
    for ti in t[1:]:
        idx = int(np.nonzero(ts32 == np.float32(ti))[0][0])
        sg = sigmas32[idx]
        an_alpha.append(float(np.float32(1.0) - sg))
        an_sigma.append(float(sg))
    return t, sig_x0, an_alpha, an_sigma


def scheduler_tables(n_train: int = 1000, shift: float = 3.0):
    """The scheduler's stored tables (fp32): sigmas [n_train + 1] ending in 0, timesteps
    [n_train] = 1000 sigma."""
    s = np.linspace(1.0, 1.0 / n_train, n_train)
    sig = shift * s / (1 + (shift - 1) * s)
    sigmas32 = np.concatenate([sig, [0.0]]).astype(np.float32)
    ts32 = (sigmas32[:-1].astype(np.float64) * 1000.0).astype(np.float32)
    return sigmas32, ts32


@dataclass(frozen=True)
class LingbotConfig:
    name: str = "lingbot_1_3b"
    dim: int = 1536
    heads: int = 12
    head_dim: int = 128
    ffn: int = 8960
    layers: int = 30
    freq_dim: int = 256
    text_len: int = 512
    text_dim: int = 4096
    lat_ch: int = 16
    y_ch: int = 20                      # image condition: 4 mask + 16 latent channels
    cam_ch: int = 384                   # Plücker: 6 channels x (8 x 8) pixels per latent pixel
    chunk: int = 4                      # latent frames per chunk
    lat_h: int = 58
    lat_w: int = 104
    local_attn: int = LOCAL_ATTN
    sink: int = SINK
    eps: float = 1e-6
    steps_index: Tuple[int, ...] = (0, 250, 500, 750)
    shift: float = 3.0

    @property
    def frame_tokens(self) -> int:
        return (self.lat_h // 2) * (self.lat_w // 2)

    @property
    def tokens(self) -> int:
        return self.chunk * self.frame_tokens

    @property
    def kv_tokens(self) -> int:
        return self.local_attn * self.frame_tokens

    def schedule(self):
        return flow_schedule(self.steps_index, 1000, self.shift)

    def replace(self, **kw) -> "LingbotConfig":
        d = dict(self.__dict__)
        d.update(kw)
        return LingbotConfig(**d)

    def flops(self) -> Dict[str, float]:
        """Algorithmic flops of one steady chunk (5 forwards + the camera branch)."""
        L, D, F, Lk, T = self.tokens, self.dim, self.ffn, self.kv_tokens, self.text_len
        per_fwd_gemm = 2.0 * L * (4 * D * D + 2 * D * D + 2 * D * F) + 2.0 * L * self.lat_ch * 4 * D
        per_fwd_attn = 4.0 * L * (Lk + T) * D
        cam = 2.0 * L * (self.cam_ch * 4 * D + 2 * D * D) + self.layers * 2.0 * L * 4 * D * D
        return {"gemm": 5 * self.layers * per_fwd_gemm, "attention": 5 * self.layers * per_fwd_attn, "camera": cam,
                "total": 5 * self.layers * (per_fwd_gemm + per_fwd_attn) + cam}


LINGBOT = LingbotConfig()
# parity-test shape: the same structure, 2 blocks, 256 wide, an 8 x 16 latent (32 tokens per frame)
LINGBOT_SMALL = LingbotConfig(name="lingbot_small", dim=256, heads=2, ffn=512, layers=2, text_dim=64, text_len=24,
                              cam_ch=24, lat_h=8, lat_w=16)


# ------------------------------------------------------------------------------ weights
def param_specs(cfg: LingbotConfig) -> List[Tuple[str, Tuple[int, ...], str]]:
    """Parameters of the DiT under the module names ``static.py`` reads (init kind last)."""
    D, F = cfg.dim, cfg.ffn
    cin = cfg.lat_ch + cfg.y_ch
    s = [("patch_embedding.weight", (D, cin, 1, 2, 2), "lin"), ("patch_embedding.bias", (D,), "bias"),
         ("text_embedding.0.weight", (D, cfg.text_dim), "lin"), ("text_embedding.0.bias", (D,), "bias"),
         ("text_embedding.2.weight", (D, D), "lin"), ("text_embedding.2.bias", (D,), "bias"),
         ("time_embedding.0.weight", (D, cfg.freq_dim), "lin"), ("time_embedding.0.bias", (D,), "bias"),
         ("time_embedding.2.weight", (D, D), "lin"), ("time_embedding.2.bias", (D,), "bias"),
         ("time_projection.1.weight", (6 * D, D), "lin"), ("time_projection.1.bias", (6 * D,), "bias"),
         ("patch_embedding_wancamctrl.weight", (D, cfg.cam_ch * 4), "lin"),
         ("patch_embedding_wancamctrl.bias", (D,), "bias"),
         ("c2ws_hidden_states_layer1.weight", (D, D), "lin"), ("c2ws_hidden_states_layer1.bias", (D,), "bias"),
         ("c2ws_hidden_states_layer2.weight", (D, D), "small"), ("c2ws_hidden_states_layer2.bias", (D,), "bias"),
         ("head.modulation", (1, 2, D), "mod"), ("head.head.weight", (cfg.lat_ch * 4, D), "lin"),
         ("head.head.bias", (cfg.lat_ch * 4,), "bias")]
    for i in range(cfg.layers):
        p = f"blocks.{i}."
        s.append((p + "modulation", (1, 6, D), "mod"))
        for m in ("self_attn", "cross_attn"):
            for n in ("q", "k", "v", "o"):
                s += [(p + f"{m}.{n}.weight", (D, D), "lin"), (p + f"{m}.{n}.bias", (D,), "bias")]
            s += [(p + f"{m}.norm_q.weight", (D,), "normw"), (p + f"{m}.norm_k.weight", (D,), "normw")]
        s += [(p + "norm3.weight", (D,), "normw"), (p + "norm3.bias", (D,), "normb"),
              (p + "ffn.0.weight", (F, D), "lin"), (p + "ffn.0.bias", (F,), "bias"),
              (p + "ffn.2.weight", (D, F), "lin"), (p + "ffn.2.bias", (D,), "bias")]
        for n in ("cam_injector_layer1", "cam_injector_layer2", "cam_scale_layer", "cam_shift_layer"):
            s += [(p + f"{n}.weight", (D, D), "small" if n in ("cam_scale_layer", "cam_shift_layer") else "lin"),
                  (p + f"{n}.bias", (D,), "bias")]
    return s


def synthetic_state_dict(cfg: LingbotConfig = LINGBOT, seed: int = 0, device="cpu") -> Dict[str, torch.Tensor]:
    """Seeded bf16 weights, one generator per tensor (the checkpoint is not available here)."""
    out = {}
    for name, shape, kind in param_specs(cfg):
        g = torch.Generator(device=device).manual_seed(
            int.from_bytes(hashlib.sha1(f"lb{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 63) - 1))
        fan_in = math.prod(shape[1:]) if len(shape) > 1 else shape[0]
        u = (torch.rand(shape, generator=g, device=device) * 2 - 1)
        if kind == "lin":
            t = u * math.sqrt(3.0 / fan_in)
        elif kind == "small":
            t = u * 0.2 * math.sqrt(3.0 / fan_in)
        elif kind == "bias":
            t = u * 0.02
        elif kind == "normw":
            t = 1 + u * 0.1
        elif kind == "normb":
            t = u * 0.1
        else:   # modulation tables
            t = torch.randn(shape, generator=g, device=device) / math.sqrt(cfg.dim)
        out[name] = t.to(torch.bfloat16)
    return out


@dataclass
class LingbotInputs:
    """A session's inputs (the reference's ``Inputs``, ``engine.py:138-142``): initial noise
    [16, lat_f, h, w] fp32, image condition y [20, lat_f, h, w] fp32, Plücker features
    [1, cam_ch, lat_f, h, w] bf16, text context [n_tokens, text_dim] bf16, generator seed."""
    noise: torch.Tensor
    y: torch.Tensor
    plucker: torch.Tensor
    context: torch.Tensor
    seed: int = 42


def synthetic_inputs(cfg: LingbotConfig, n_chunks: int, seed: int = 0, text_tokens: int = None) -> LingbotInputs:
    g = torch.Generator().manual_seed(seed)
    lf = cfg.chunk * n_chunks
    noise = torch.randn(cfg.lat_ch, lf, cfg.lat_h, cfg.lat_w, generator=g)
    msk = torch.zeros(4, lf, cfg.lat_h, cfg.lat_w)
    msk[:, 0] = 1
    y = torch.cat([msk, torch.randn(cfg.y_ch - 4, lf, cfg.lat_h, cfg.lat_w, generator=g)], 0)
    pl = (torch.randn(1, cfg.cam_ch, lf, cfg.lat_h, cfg.lat_w, generator=g) * 0.5).to(torch.bfloat16)
    n_txt = text_tokens if text_tokens is not None else max(1, cfg.text_len // 2)
    ctx = torch.randn(n_txt, cfg.text_dim, generator=g).to(torch.bfloat16)
    return LingbotInputs(noise=noise, y=y, plucker=pl, context=ctx, seed=seed + 1)


# ------------------------------------------------------------------------------ engine
def pack_weights(cfg: LingbotConfig, sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Engine tensor names (``fw_lb_*``) of a state dict under the module names of
    :func:`param_specs`: q / k / v and cross k / v packed along rows, the patch embedding
    flattened to [dim, channels * 4] in (channel, dy, dx) order."""
    D = cfg.dim
    w = lambda n: sd[n].detach().to(torch.bfloat16).cpu()   # noqa: E731
    out = {"patch.w": w("patch_embedding.weight").reshape(D, -1), "patch.b": w("patch_embedding.bias"),
           "text.0.w": w("text_embedding.0.weight"), "text.0.b": w("text_embedding.0.bias"),
           "text.2.w": w("text_embedding.2.weight"), "text.2.b": w("text_embedding.2.bias"),
           "time.0.w": w("time_embedding.0.weight"), "time.0.b": w("time_embedding.0.bias"),
           "time.2.w": w("time_embedding.2.weight"), "time.2.b": w("time_embedding.2.bias"),
           "tproj.w": w("time_projection.1.weight"), "tproj.b": w("time_projection.1.bias"),
           "cam.in.w": w("patch_embedding_wancamctrl.weight"), "cam.in.b": w("patch_embedding_wancamctrl.bias"),
           "cam.h1.w": w("c2ws_hidden_states_layer1.weight"), "cam.h1.b": w("c2ws_hidden_states_layer1.bias"),
           "cam.h2.w": w("c2ws_hidden_states_layer2.weight"), "cam.h2.b": w("c2ws_hidden_states_layer2.bias"),
           "head.mod": w("head.modulation").reshape(2, D), "head.w": w("head.head.weight"),
           "head.b": w("head.head.bias"),
           "mods": torch.stack([w(f"blocks.{i}.modulation").reshape(6, D) for i in range(cfg.layers)])}
    for i in range(cfg.layers):
        b, p = f"blocks.{i}.", f"b{i}."
        sa, ca = b + "self_attn.", b + "cross_attn."
        out[p + "sa.qkv.w"] = torch.cat([w(sa + n + ".weight") for n in "qkv"])
        out[p + "sa.qkv.b"] = torch.cat([w(sa + n + ".bias") for n in "qkv"])
        out[p + "sa.o.w"], out[p + "sa.o.b"] = w(sa + "o.weight"), w(sa + "o.bias")
        out[p + "sa.nq.w"], out[p + "sa.nk.w"] = w(sa + "norm_q.weight"), w(sa + "norm_k.weight")
        out[p + "n3.w"], out[p + "n3.b"] = w(b + "norm3.weight"), w(b + "norm3.bias")
        out[p + "ca.q.w"], out[p + "ca.q.b"] = w(ca + "q.weight"), w(ca + "q.bias")
        out[p + "ca.kv.w"] = torch.cat([w(ca + "k.weight"), w(ca + "v.weight")])
        out[p + "ca.kv.b"] = torch.cat([w(ca + "k.bias"), w(ca + "v.bias")])
        out[p + "ca.o.w"], out[p + "ca.o.b"] = w(ca + "o.weight"), w(ca + "o.bias")
        out[p + "ca.nq.w"], out[p + "ca.nk.w"] = w(ca + "norm_q.weight"), w(ca + "norm_k.weight")
        out[p + "ffn.0.w"], out[p + "ffn.0.b"] = w(b + "ffn.0.weight"), w(b + "ffn.0.bias")
        out[p + "ffn.2.w"], out[p + "ffn.2.b"] = w(b + "ffn.2.weight"), w(b + "ffn.2.bias")
        for m, n in (("inj1", "cam_injector_layer1"), ("inj2", "cam_injector_layer2"), ("scale", "cam_scale_layer"),
                     ("shift", "cam_shift_layer")):
            out[p + f"cam.{m}.w"], out[p + f"cam.{m}.b"] = w(b + n + ".weight"), w(b + n + ".bias")
    return out


def make_config(cfg: LingbotConfig):
    from . import _lib
    c = _lib.FwLbConfig()
    for f in ("dim", "heads", "head_dim", "ffn", "layers", "freq_dim", "text_len", "text_dim", "lat_ch", "y_ch",
              "cam_ch", "chunk", "lat_h", "lat_w"):
        setattr(c, f, getattr(cfg, f))
    c.kv_frames, c.sink_frames, c.eps = cfg.local_attn, cfg.sink, cfg.eps
    t, sig_x0, an_alpha, an_sigma = cfg.schedule()
    c.n_steps = len(t)
    for i, v in enumerate(t):
        c.timesteps[i] = v
        c.sig_x0[i] = sig_x0[i]
    for i, (a, s) in enumerate(zip(an_alpha, an_sigma)):
        c.an_alpha[i], c.an_sigma[i] = a, s
    return c


class B200StaticLingbot:
    """The LingBot causal runtime on one GPU, with the reference ``StaticLingbot``'s methods
    (``static.py:49-320``): ``set_prompt``, ``set_session``, ``reset``, ``keys``, ``capture``,
    ``gen_chunk(k, graph, cam)``, ``state`` / ``load`` / ``state_bytes``.

    ``weights``: a state dict under :func:`param_specs` names (``None`` = seeded synthetic).
    One library-held CUDA graph serves every chunk: the chunk's plan and index are written to
    device buffers before the replay."""

    def __init__(self, cfg: LingbotConfig = LINGBOT, weights=None, device="cuda", seed: int = 0,
                 max_chunks: int = 4096):
        import ctypes

        from . import _lib
        from ._lib import check, lib, ptr
        self.cfg = cfg
        self.dev = torch.device(device)
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        sd = synthetic_state_dict(cfg, seed) if weights is None else weights
        packed = pack_weights(cfg, sd)
        self._lib = lib()
        self._ccfg = make_config(cfg)
        self.plans = chunk_plans(max_chunks, cfg.chunk, cfg.local_attn, cfg.sink)
        dt = {_lib.DT_BF16: torch.bfloat16, _lib.DT_F32: torch.float32, _lib.DT_I32: torch.int32,
              _lib.DT_U8: torch.uint8}
        with torch.cuda.device(self.dev):
            h = ctypes.c_void_p()
            check(self._lib.fw_lb_create(ctypes.byref(self._ccfg), ctypes.byref(h)), "fw_lb_create")
            self._h = h
            self.buffers: Dict[str, torch.Tensor] = {}
            for i in range(self._lib.fw_lb_tensor_count(h)):
                info = _lib.FwTensorInfo()
                check(self._lib.fw_lb_tensor_info_at(h, i, ctypes.byref(info)), "fw_lb_tensor_info_at")
                name, shape = info.name.decode(), tuple(info.shape[j] for j in range(info.ndim))
                if info.kind == _lib.KIND_WEIGHT:
                    w = packed[name]
                    if tuple(w.shape) != shape:
                        raise ValueError(f"weight {name}: shape {tuple(w.shape)} != {shape}")
                    t = w.to(self.dev).contiguous()
                else:
                    t = torch.zeros(shape, dtype=dt[info.dtype], device=self.dev)
                self.buffers[name] = t
                check(self._lib.fw_lb_bind(h, name.encode(), ptr(t), t.numel() * t.element_size()),
                      f"fw_lb_bind({name})")
            check(self._lib.fw_lb_finalize(h), "fw_lb_finalize")
            torch.cuda.synchronize(self.dev)
        B = self.buffers
        self.K = [B[f"K.{i}"] for i in range(cfg.layers)]
        self.V = [B[f"V.{i}"] for i in range(cfg.layers)]
        self.x_in, self.y_in, self.pl_in, self.out = B["x_in"], B["y_in"], B["pl_in"], B["out"]
        self.noise = [B[f"noise.{i}"] for i in range(len(cfg.steps_index) - 1)]
        self.graph, self.I, self.live = None, None, 0
        self.g = None

    # ------------------------------------------------------------------ session
    def set_prompt(self, context: torch.Tensor) -> None:
        """Text embedding and every block's cross-attention K/V of a prompt (``static.py:128-137``)."""
        from ._lib import check, stream_ptr
        c = self.cfg
        ctx = self.buffers["ctx_in"]
        ctx.zero_()
        ctx[:context.shape[0]].copy_(context)
        with torch.cuda.device(self.dev):
            check(self._lib.fw_lb_set_prompt(self._h, stream_ptr()), "fw_lb_set_prompt")

    def set_session(self, I: LingbotInputs) -> None:
        if self.I is None or self.I.context is not I.context:
            self.set_prompt(I.context.to(self.dev))
        self.I = I
        self.noise_all = I.noise.to(self.dev, torch.float32)
        self.y_all = I.y.to(self.dev, torch.float32)
        self.pl_all = I.plucker.to(self.dev, torch.bfloat16)
        self.reset()

    def reset(self) -> None:
        for t in self.K + self.V:
            t.zero_()
        self.live = 0
        self.g = torch.Generator(device=self.dev)
        self.g.manual_seed(self.I.seed if self.I is not None else 0)

    def keys(self):
        return sorted(set(self.plans[:16]), key=lambda p: (p[1], p[0]))

    def _prep(self, k: int, cam=None, noise: bool = True) -> None:
        """Chunk inputs (``static.py:154-169``) and the chunk's device plan."""
        c = self.cfg
        s = c.chunk * k
        self.x_in.copy_(self.noise_all[:, s:s + c.chunk])
        self.y_in.copy_(self.y_all[:, s:s + c.chunk])
        self.pl_in.copy_(self.pl_all[0, :, s:s + c.chunk] if cam is None else cam.reshape(self.pl_in.shape))
        if noise:
            for nb in self.noise:
                nb.copy_(torch.randn(nb.shape, generator=self.g, device=self.dev, dtype=torch.float32))
        woff, klen, roll = self.plans[k]
        Ft = c.frame_tokens
        src, dst, n = roll if roll is not None else (0, 0, 0)
        plan = [woff * Ft, klen * Ft, 0, src * Ft, dst * Ft, n * Ft, (src - dst) * Ft, 0]
        self.buffers["plan"].copy_(torch.tensor(plan, dtype=torch.int32))
        self.buffers["chunk"].copy_(torch.tensor([k, s, 0, 0], dtype=torch.int32))

    def _launch(self) -> None:
        from ._lib import check, stream_ptr
        check(self._lib.fw_lb_chunk(self._h, stream_ptr()), "fw_lb_chunk")

    def capture(self, warmup: int = 0) -> None:
        """One library-held graph for every plan (the plan is read on the device); recording
        runs nothing, so the session state is unchanged."""
        from .graph import LibGraph
        with torch.cuda.device(self.dev):
            self.graph = LibGraph.record(self._launch)

    @torch.no_grad()
    def gen_chunk(self, k: int, graph: bool = True, cam=None) -> torch.Tensor:
        """x0 of chunk k, [16, C, h, w] fp32 (``static.py:296-305``)."""
        with torch.cuda.device(self.dev):
            self._prep(k, cam=cam)
            if graph:
                if self.graph is None:
                    self.capture()
                self.graph.replay()
            else:
                self._launch()
            woff, klen, roll = self.plans[k]
            self.live = klen if roll is None else roll[1] + roll[2]
            return self.out.clone()

    # ------------------------------------------------------------------ state
    def state(self):
        n = self.live * self.cfg.frame_tokens
        return dict(kv=[t[:n].clone() for t in self.K + self.V], live=self.live, g=self.g.get_state())

    def load(self, st) -> None:
        n = st["live"] * self.cfg.frame_tokens
        for d, s in zip(self.K + self.V, st["kv"]):
            d[:n].copy_(s, non_blocking=True)
        self.live = st["live"]
        self.g.set_state(st["g"])

    def state_bytes(self, live=None) -> int:
        live = self.live if live is None else live
        return sum(t[:live * self.cfg.frame_tokens].numel() * t.element_size() for t in self.K + self.V)

    def device_status(self) -> int:
        return int(self.buffers["status"][0])

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and getattr(self, "_lib", None) is not None:
            self.graph = None
            self._lib.fw_lb_destroy(h)
            self._h = None
