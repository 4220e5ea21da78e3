"""Host-side chunk preparation: action windows, path seeds, synthetic images, noise.

Restates the semantics of ``StaticMG._prep`` (``fastworld/models/mg2/static.py:76-127``) and
``path_seed`` (``fastworld/models/mg2/model.py:25-26``).  A path is a list of chunk keys
``(image_name, (keyboard, mouse))``; keyboard/mouse are either names from ``KEYS``/``CAM``
(``model.py:21-22``) or explicit vectors (4-dim multi-hot keyboard, 2-dim mouse).
"""
from __future__ import annotations

import hashlib
from typing import Dict, List, Sequence, Tuple

import torch

KEYS = {"w": (1, 0, 0, 0), "s": (0, 1, 0, 0), "a": (0, 0, 1, 0), "d": (0, 0, 0, 1), "q": (0, 0, 0, 0)}
CAM = {"i": (0.1, 0), "k": (-0.1, 0), "j": (0, -0.1), "l": (0, 0.1), "u": (0, 0)}


def path_seed(path) -> int:
    """Seed of a path prefix: the low 63 bits of sha1(repr(tuple(path))) (model.py:25-26)."""
    return int.from_bytes(hashlib.sha1(repr(tuple(path)).encode()).digest()[:8], "little") & ((1 << 63) - 1)


def _vec(table, a) -> Tuple[float, ...]:
    return tuple(table[a]) if isinstance(a, str) else tuple(float(v) for v in a)


def chunk_of_pixel_frame(q: int, frames: int, ratio: int) -> int:
    """Chunk that owns pixel frame q: chunk 0 has 1 + ratio*(frames-1) pixel frames, later
    chunks ratio*frames each (model.py:73-79)."""
    first = 1 + ratio * (frames - 1)
    return 0 if q < first else 1 + (q - first) // (ratio * frames)


def action_windows(cfg, path: Sequence, k: int):
    """Keyboard window ``kc`` [kc_len, 4] and grouped mouse window ``gm`` [frames, pad_t, 2]
    read by the action module at chunk k, as bf16 tensors (static.py:85-112).

    The action module sees the padded per-pixel-frame action sequence (``pad_t`` copies of
    the first action, then one action per pixel frame) from position ratio*frames*k on;
    frame f of the chunk reads the ``pad_t`` entries starting at ratio*f."""
    r, F, pad = cfg.time_ratio, cfg.frames, cfg.pad_t
    start = r * F * k
    kb, ms = [], []
    for i in range(cfg.kc_len):
        q = start + i - pad
        j = 0 if q < 0 else chunk_of_pixel_frame(q, F, r)
        kb.append(_vec(KEYS, path[j][1][0]))
        ms.append(_vec(CAM, path[j][1][1]))
    kc = torch.tensor(kb, dtype=torch.float32).to(torch.bfloat16)
    mc = torch.tensor(ms, dtype=torch.float32).to(torch.bfloat16)
    gm = torch.stack([mc[r * f: r * f + pad] for f in range(F)], 0)
    return kc, gm


def window_chunks(cfg, k: int) -> Tuple[int, int]:
    """First and last chunk whose actions the action module's window at chunk k reads."""
    r, F, pad = cfg.time_ratio, cfg.frames, cfg.pad_t
    lo, hi = r * F * k - pad, r * F * k + cfg.kc_len - 1 - pad
    j = lambda q: 0 if q < 0 else chunk_of_pixel_frame(q, F, r)  # noqa: E731
    return j(lo), j(hi)


def device_prep_actions(cfg, path: Sequence, k: int) -> Tuple[int, List[Tuple[float, ...]]]:
    """(j_lo, per-chunk action vectors) that ``fw_prep`` needs for chunk k: keyboard then mouse
    values of chunks j_lo .. (the last chunk the window reads)."""
    lo, hi = window_chunks(cfg, k)
    return lo, [_vec(KEYS, path[j][1][0]) + _vec(CAM, path[j][1][1]) for j in range(lo, hi + 1)]


def synthetic_image(cfg, seed: int, max_chunks: int = 24, device="cpu") -> Dict[str, torch.Tensor]:
    """A seeded stand-in for ``Model.add_image`` (model.py:53-68): ``cond_concat`` = 4 mask
    channels (1 on the first latent frame) + 16 N(0,1) latent channels, ``visual_context`` =
    N(0,1) CLIP tokens.  Both bf16."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    nf = cfg.frames * max_chunks
    lat = torch.randn(1, cfg.cond_ch - 4, nf, cfg.lat_h, cfg.lat_w, generator=g)
    mask = torch.zeros(1, 4, nf, cfg.lat_h, cfg.lat_w)
    mask[:, :, 0] = 1
    vis = torch.randn(1, cfg.ctx_tokens, cfg.ctx_dim, generator=g)
    return {"cond_concat": torch.cat([mask, lat], 1).to(torch.bfloat16).to(device),
            "visual_context": vis.to(torch.bfloat16).to(device)}


def draw_noise(cfg, path: Sequence, k: int, device="cpu") -> List[torch.Tensor]:
    """Initial latent and the per-step renoising noise of chunk k, drawn in the eager order
    from a generator seeded with ``path_seed(path[:k+1])`` (static.py:124-127, model.py:102-109).
    Returns [x_in [1,16,F,H,W]] + (n_steps - 1) x [F,16,H,W], bf16."""
    g = torch.Generator(device=device).manual_seed(path_seed(path[:k + 1]))
    F, H, W = cfg.frames, cfg.lat_h, cfg.lat_w
    out = [torch.randn((1, cfg.lat_ch, F, H, W), generator=g, device=device, dtype=torch.bfloat16)]
    for _ in range(len(cfg.steps) - 1):
        out.append(torch.randn((F, cfg.lat_ch, H, W), generator=g, device=device, dtype=torch.bfloat16))
    return out
