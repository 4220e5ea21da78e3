"""CPU oracle for the streaming TAEHV decoder.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it.  The product path (``fastworld_b200.vae``) runs the
sm_100a kernels of ``csrc/taehv.cu`` and fails loudly when its CUDA library is missing.

What it restates: the reference's ``TinyVAE`` (``fastworld/models/mg2/vae.py:95-124``) calls the
third-party TAEHV package (github.com/madebyollin/taehv, ``taew2_1.pth``; cloned unpinned by
``docs/setup.md:39``, absent from the reference tree) through its ``StreamingTAEHV`` wrapper:
``decode`` feeds one latent chunk and drains every frame it yields, the first ``frames_to_trim``
frames of a stream are dropped, and the output is mapped to [-1, 1] by ``x * 2 - 1``
(``vae.py:100-109``); the state is the MemBlocks' memory plus the count of decoded frames
(``vae.py:112-119``).  The decoder itself is restated from TAEHV's published architecture, in
fp32 NCHW with ``torch.nn.functional``, frame-parallel within a chunk:

* :func:`clamp`        Clamp:  3 tanh(x / 3)
* :func:`memblock`     MemBlock: ReLU(conv(ReLU(conv(ReLU(conv(cat[x, past]))))) + x); ``past`` is
                       the block's input one frame earlier, the carried state for a chunk's
                       first frame (zeros at the start of a stream)
* :func:`tgrow`        TGrow: 1 x 1 conv C -> C r, output channels [j C, (j + 1) C) of frame f
                       become frame f r + j
* :meth:`TaehvOracle.decode`  the whole decoder and the streaming wrapper's trim

Parity: unpinned against TAEHV itself (its code and checkpoint are not available here); the
oracle and the engine share only the architecture above and the checkpoint key names.  The
streaming form is checked against the whole-sequence form of the same decoder
(``tests/test_taehv_host.py``): chunked decoding with carried memory equals decoding all frames
at once, as StreamingTAEHV's contract requires.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn.functional as F


def clamp(x: torch.Tensor) -> torch.Tensor:
    return torch.tanh(x / 3) * 3


def conv(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    return F.conv2d(x, w, b, padding=w.shape[-1] // 2)


def memblock(sd: Dict[str, torch.Tensor], p: str, x: torch.Tensor, mem: torch.Tensor) -> torch.Tensor:
    """x: [T, C, H, W] frames of one chunk; mem: [C, H, W] the input frame before x[0]."""
    past = torch.cat([mem[None], x[:-1]], 0)
    y = F.relu(conv(torch.cat([x, past], 1), sd[f"{p}.0.weight"], sd[f"{p}.0.bias"]))
    y = F.relu(conv(y, sd[f"{p}.2.weight"], sd[f"{p}.2.bias"]))
    y = conv(y, sd[f"{p}.4.weight"], sd[f"{p}.4.bias"])
    return F.relu(y + x)


def tgrow(x: torch.Tensor, w: torch.Tensor, r: int) -> torch.Tensor:
    T, C, H, W = x.shape
    return conv(x, w).reshape(T * r, C, H, W)


class TaehvOracle:
    """fp32 streaming decoder over a TAEHV decoder state dict (any float dtype; used in fp32)."""

    def __init__(self, cfg, sd: Dict[str, torch.Tensor]):
        self.cfg = cfg
        self.sd = {k: v.float() for k, v in sd.items()}
        self.reset()

    def reset(self) -> None:
        self.mem: List[Optional[torch.Tensor]] = [None] * 9
        self.n_frames_decoded = 0

    def decoder(self, lat: torch.Tensor) -> torch.Tensor:
        """lat [16, T, h, w] -> frames [T * prod(time_up), 3, 8h, 8w] in [0, 1]; updates memory."""
        sd, cfg = self.sd, self.cfg
        x = clamp(lat.float().transpose(0, 1))
        x = F.relu(conv(x, sd["decoder.1.weight"], sd["decoder.1.bias"]))
        for s in range(3):
            b = 3 + 6 * s
            for k in range(3):
                i = 3 * s + k
                mem = self.mem[i] if self.mem[i] is not None else torch.zeros_like(x[0])
                self.mem[i] = x[-1].clone()
                x = memblock(sd, f"decoder.{b + k}.conv", x, mem)
            x = F.interpolate(x, scale_factor=2, mode="nearest")
            x = tgrow(x, sd[f"decoder.{b + 4}.conv.weight"], cfg.time_up[s])
            x = conv(x, sd[f"decoder.{b + 5}.weight"])
        x = conv(F.relu(x), sd["decoder.22.weight"], sd["decoder.22.bias"])
        return x.clamp(0, 1)

    def decode(self, lat: torch.Tensor) -> torch.Tensor:
        """One chunk as ``TinyVAE.decode``: frames in [-1, 1], the stream's first frames trimmed."""
        if lat.dim() == 5:
            lat = lat[0]
        x = self.decoder(lat)
        if self.n_frames_decoded == 0:
            x = x[self.cfg.trim:]
        self.n_frames_decoded += x.shape[0]
        return x * 2 - 1

    def state(self):
        return [m.clone() if m is not None else None for m in self.mem], self.n_frames_decoded

    def load(self, st) -> None:
        mem, n = st
        self.mem = [m.clone() if m is not None else None for m in mem]
        self.n_frames_decoded = n
