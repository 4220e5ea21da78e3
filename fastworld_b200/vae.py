"""Streaming TAEHV decoder on the engine's sm_100a kernels: the reference's ``TinyVAE``
(``fastworld/models/mg2/vae.py:95-124``) with the same methods and contracts.

``TinyVAE.decode(lat)`` turns one MG2 latent chunk [1, 16, 3, 44, 80] into RGB frames
[T, 3, 352, 640] fp32 in [-1, 1] on the GPU (T = 9 for a stream's first chunk, 12 after: the
decoder emits 4 frames per latent frame and drops the first 3 of a stream, TAEHV's
``frames_to_trim``).  ``reset`` starts a new stream, ``state`` / ``load`` save and restore it
(``vae.py:112-119``), ``state_bytes`` is its size.

The decoder is TAEHV (github.com/madebyollin/taehv, checkpoint ``taew2_1.pth``), a third-party
package that the reference clones unpinned (``docs/setup.md:39``) and that is not part of the
reference tree.  Its decoder, restated from the published architecture:

    Clamp(3 tanh(x / 3)), conv3x3(16 -> C0) + ReLU,
    per stage s = 0, 1, 2:  3 x MemBlock(C_s), Upsample(2x nearest), TGrow(C_s, r_s),
                            conv3x3(C_s -> C_{s+1}, no bias)
    ReLU, conv3x3(C3 -> 3); output clamped to [0, 1]

with MemBlock(x, past) = ReLU(conv(ReLU(conv(ReLU(conv(cat[x, past]))))) + x), ``past`` the
block's input one frame earlier (zeros before a stream's first frame), and TGrow a bias-free
1 x 1 conv C -> C r whose output is split along channels into r consecutive frames.  taew2_1:
C = (256, 128, 64, 64), r = (1, 2, 2).

Weights are read from a TAEHV state dict (keys ``decoder.<i>...`` of its ``nn.Sequential``; see
:func:`param_specs`) or drawn by :func:`synthetic_state_dict` (the checkpoint is not available
here), rounded to fp16 like the reference's ``.to(dev, torch.float16)``.
"""
from __future__ import annotations

import ctypes
import hashlib
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_ptr


@dataclass(frozen=True)
class TaehvConfig:
    name: str = "taew2_1"
    lat_ch: int = 16
    lat_frames: int = 3                       # latent frames per chunk
    lat_h: int = 44
    lat_w: int = 80
    channels: Tuple[int, int, int, int] = (256, 128, 64, 64)
    time_up: Tuple[int, int, int] = (1, 2, 2)

    @property
    def frames_per_latent(self) -> int:
        return math.prod(self.time_up)

    @property
    def frames_out(self) -> int:
        """Frames one chunk decodes to (before the stream's first-chunk trim)."""
        return self.lat_frames * self.frames_per_latent

    @property
    def trim(self) -> int:
        """Frames dropped at the start of a stream (TAEHV frames_to_trim)."""
        return self.frames_per_latent - 1

    def stage(self, s: int) -> Tuple[int, int, int, int]:
        """(channels, frames, height, width) of stage s's MemBlocks."""
        f = self.lat_frames
        for i in range(s):
            f *= self.time_up[i]
        return self.channels[s], f, self.lat_h << s, self.lat_w << s

    def state_bytes(self) -> int:
        """fp16 bytes of the streaming state: each MemBlock's last input frame."""
        return sum(3 * c * h * w * 2 for c, _, h, w in (self.stage(s) for s in range(3)))

    def flops(self) -> float:
        """Algorithmic flops (2 per multiply-add) of one chunk: the convolutions at their output
        sizes, TGrow at the pre-upsample size (it commutes with nearest upsampling), 3 RGB
        outputs of the last conv."""
        c0, f0, h0, w0 = self.stage(0)
        fl = 2.0 * f0 * h0 * w0 * c0 * self.lat_ch * 9
        for s in range(3):
            c, f, h, w = self.stage(s)
            px, r = f * h * w, self.time_up[s]
            fl += 2.0 * px * 9 * c * (2 * c + c + c) * 3       # three MemBlocks
            fl += 2.0 * px * c * c * r                         # TGrow
            fl += 2.0 * (4 * px * r) * self.channels[s + 1] * 9 * c
        fl += 2.0 * self.frames_out * (self.lat_h * 8) * (self.lat_w * 8) * 3 * 9 * self.channels[3]
        return fl


TAEW2_1 = TaehvConfig()
# parity-test shape: the same layer structure at 64 channels on an 8 x 16 latent
TAEHV_SMALL = TaehvConfig(name="taehv_small", lat_frames=2, lat_h=8, lat_w=16, channels=(64, 64, 64, 64))


def _stage_base(s: int) -> int:
    return 3 + 6 * s        # decoder.<3 + 6 s + k> = MemBlock k, + 4 = TGrow, + 5 = conv


def param_specs(cfg: TaehvConfig) -> List[Tuple[str, Tuple[int, ...], str]]:
    """TAEHV decoder parameters (name, shape, init kind) under the checkpoint's key names."""
    C = cfg.channels
    out = [("decoder.1.weight", (C[0], cfg.lat_ch, 3, 3), "relu"), ("decoder.1.bias", (C[0],), "bias")]
    for s in range(3):
        b = _stage_base(s)
        for k in range(3):
            p = f"decoder.{b + k}.conv"
            out += [(f"{p}.0.weight", (C[s], 2 * C[s], 3, 3), "relu"), (f"{p}.0.bias", (C[s],), "bias"),
                    (f"{p}.2.weight", (C[s], C[s], 3, 3), "relu"), (f"{p}.2.bias", (C[s],), "bias"),
                    (f"{p}.4.weight", (C[s], C[s], 3, 3), "resid"), (f"{p}.4.bias", (C[s],), "bias")]
        out.append((f"decoder.{b + 4}.conv.weight", (C[s] * cfg.time_up[s], C[s], 1, 1), "linear"))
        out.append((f"decoder.{b + 5}.weight", (C[s + 1], C[s], 3, 3), "relu" if s == 2 else "linear"))
    out += [("decoder.22.weight", (3, C[3], 3, 3), "out"), ("decoder.22.bias", (3,), "out_bias")]
    return out


def synthetic_state_dict(cfg: TaehvConfig = TAEW2_1, seed: int = 0) -> Dict[str, torch.Tensor]:
    """Seeded TAEHV decoder weights (fp16, CPU), one generator per tensor: He-scaled convs before
    ReLUs, half-scale residual branches, an output layer whose values fall mostly inside [0, 1]
    so that the final clamp is exercised but not saturated."""
    sd = {}
    for name, shape, kind in param_specs(cfg):
        g = torch.Generator().manual_seed(int.from_bytes(hashlib.sha1(f"{seed}:{name}".encode()).digest()[:8],
                                                         "little") & ((1 << 63) - 1))
        fan_in = math.prod(shape[1:]) if len(shape) > 1 else 1
        t = torch.randn(shape, generator=g)
        if kind == "relu":
            t *= math.sqrt(2.0 / fan_in)
        elif kind == "resid":
            t *= 0.5 * math.sqrt(1.0 / fan_in)
        elif kind == "linear":
            t *= math.sqrt(1.0 / fan_in)
        elif kind == "out":
            t *= 0.25 * math.sqrt(1.0 / fan_in)
        elif kind == "bias":
            t *= 0.05
        elif kind == "out_bias":
            t = 0.3 + 0.05 * t
        sd[name] = t.to(torch.float16)
    return sd


def _conv_k(w: torch.Tensor) -> torch.Tensor:
    """[Cout, Cin, kh, kw] -> [Cout, kh * kw * Cin] with K ordered (tap, input channel)."""
    return w.permute(0, 2, 3, 1).reshape(w.shape[0], -1)


def pack_weights(cfg: TaehvConfig, sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Device layouts (fw_taehv tensor names) of a TAEHV decoder state dict: fp16 weights
    [Cout, taps * Cin], fp32 biases (the fp16 values, widened)."""
    h = lambda t: t.detach().to(torch.float16).cpu()            # noqa: E731
    f = lambda t: t.detach().to(torch.float16).float().cpu()    # noqa: E731
    out = {}
    w = _conv_k(h(sd["decoder.1.weight"]))
    out["conv_in.w"] = torch.cat([w, torch.zeros(w.shape[0], 192 - w.shape[1], dtype=w.dtype)], 1)
    out["conv_in.b"] = f(sd["decoder.1.bias"])
    for s in range(3):
        b = _stage_base(s)
        for k in range(3):
            p, q = f"decoder.{b + k}.conv", f"mb{3 * s + k}"
            for j, i in enumerate((0, 2, 4)):
                out[f"{q}.w{j}"] = _conv_k(h(sd[f"{p}.{i}.weight"]))
                out[f"{q}.b{j}"] = f(sd[f"{p}.{i}.bias"])
        out[f"tgrow{s}.w"] = _conv_k(h(sd[f"decoder.{b + 4}.conv.weight"]))
        out[f"conv{s}.w"] = _conv_k(h(sd[f"decoder.{b + 5}.weight"]))
    # the last conv, transposed: row (ky * 3 + kx) * 3 + c holds W[c, :, ky, kx]
    w = h(sd["decoder.22.weight"]).permute(2, 3, 0, 1).reshape(27, -1)
    out["conv_out.wt"] = torch.cat([w, torch.zeros(32 - w.shape[0], w.shape[1], dtype=w.dtype)], 0)
    out["conv_out.b"] = torch.cat([f(sd["decoder.22.bias"]), torch.zeros(29)])
    return out


def make_config(cfg: TaehvConfig) -> _lib.FwTaehvConfig:
    c = _lib.FwTaehvConfig()
    c.lat_ch, c.lat_frames, c.lat_h, c.lat_w = cfg.lat_ch, cfg.lat_frames, cfg.lat_h, cfg.lat_w
    for i in range(4):
        c.channels[i] = cfg.channels[i]
    for i in range(3):
        c.time_up[i] = cfg.time_up[i]
    return c


_DT = {_lib.DT_BF16: torch.bfloat16, _lib.DT_F32: torch.float32, _lib.DT_F16: torch.float16, _lib.DT_I32: torch.int32,
       _lib.DT_U8: torch.uint8}


class TinyVAE:
    """TAEHV streaming decoder on one GPU (``fastworld/models/mg2/vae.py:95-124``).

    ``ckpt``: a TAEHV state dict (or a path to one) for the real weights; ``None`` draws
    :func:`synthetic_state_dict` with ``seed``.  Every ``decode`` replays one CUDA graph held by
    the library (recorded on the first call) unless ``use_graph`` is False."""

    def __init__(self, dev="cuda", ckpt=None, cfg: TaehvConfig = TAEW2_1, seed: int = 0, use_graph: bool = True):
        self.dev = torch.device(dev)
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        self.cfg, self.use_graph = cfg, use_graph
        if isinstance(ckpt, str):
            ckpt = torch.load(ckpt, map_location="cpu")
        sd = synthetic_state_dict(cfg, seed) if ckpt is None else ckpt
        packed = pack_weights(cfg, sd)
        self._lib = lib()
        self._ccfg = make_config(cfg)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.dev):
            check(self._lib.fw_taehv_create(ctypes.byref(self._ccfg), ctypes.byref(h)), "fw_taehv_create")
            self._h = h
            self.buffers: Dict[str, torch.Tensor] = {}
            for i in range(self._lib.fw_taehv_tensor_count(h)):
                info = _lib.FwTensorInfo()
                check(self._lib.fw_taehv_tensor_info_at(h, i, ctypes.byref(info)), "fw_taehv_tensor_info_at")
                name, shape = info.name.decode(), tuple(info.shape[j] for j in range(info.ndim))
                dt = _DT[info.dtype]
                if info.kind == _lib.KIND_WEIGHT:
                    w = packed[name]
                    if tuple(w.shape) != shape:
                        raise ValueError(f"weight {name}: shape {tuple(w.shape)} != {shape}")
                    t = w.to(self.dev, dt).contiguous()
                else:
                    t = torch.zeros(shape, dtype=dt, device=self.dev)
                self.buffers[name] = t
                check(self._lib.fw_taehv_bind(h, name.encode(), ptr(t), t.numel() * t.element_size()),
                      f"fw_taehv_bind({name})")
            check(self._lib.fw_taehv_finalize(h), "fw_taehv_finalize")
            torch.cuda.synchronize(self.dev)
        self.lat, self.rgb, self.mem = self.buffers["lat"], self.buffers["rgb"], self.buffers["mem"]
        self.n_frames_decoded = 0
        self.graph = None

    # ------------------------------------------------------------------ decoding
    def _launch(self) -> None:
        check(self._lib.fw_taehv_decode(self._h, stream_ptr()), "fw_taehv_decode")

    def capture(self) -> None:
        """Record the decoder's launches as one library-held CUDA graph (runs nothing)."""
        from .graph import LibGraph
        with torch.cuda.device(self.dev):
            self.graph = LibGraph.record(self._launch)

    @torch.no_grad()
    def decode(self, lat: torch.Tensor, graph: Optional[bool] = None) -> torch.Tensor:
        """lat: [1, 16, F, h, w] or [16, F, h, w] (any float dtype; cast to fp16 as the reference
        does).  Returns frames [T, 3, 8h, 8w] fp32 in [-1, 1] on the GPU."""
        graph = self.use_graph if graph is None else graph
        if lat.dim() == 5:
            lat = lat[0]
        with torch.cuda.device(self.dev):
            self.lat.copy_(lat)
            if graph:
                if self.graph is None:
                    self.capture()
                self.graph.replay()
            else:
                self._launch()
            out = self.rgb
            if self.n_frames_decoded == 0:
                out = out[self.cfg.trim:]
            self.n_frames_decoded += out.shape[0]
            return out.clone()

    # ------------------------------------------------------------------ streaming state
    def reset(self) -> None:
        self.mem.zero_()
        self.n_frames_decoded = 0

    def state(self):
        return self.mem.clone(), self.n_frames_decoded

    def load(self, st) -> None:
        mem, n = st
        self.mem.copy_(mem, non_blocking=True)
        self.n_frames_decoded = n

    def state_bytes(self) -> int:
        return self.mem.numel() * self.mem.element_size()

    def device_status(self) -> int:
        out = ctypes.c_int()
        check(self._lib.fw_taehv_status(self._h, ctypes.byref(out)), "fw_taehv_status")
        return out.value

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and getattr(self, "_lib", None) is not None:
            self.graph = None
            self._lib.fw_taehv_destroy(h)
            self._h = None
