"""CPU restatement of the device chunk preparation's noise.  TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module; the product path draws its noise on the GPU
(``fw_prep``, fastworld_b200/csrc/prep.cu) or with torch.randn on the host path.

Philox-4x32-10 is the counter-based generator of Salmon, Moraes, Dror and Shaw ("Parallel
random numbers: as easy as 1, 2, 3", SC 2011); ``PHILOX_KAT`` holds three of the known-answer
vectors published with it (Random123's ``kat_vectors``), which pin this restatement and the
library's generator.  The noise layout is the one ``fw_prep`` defines: key = the 64-bit path
seed (``path_seed``, fastworld/models/mg2/model.py:25-26), counter = {group, tensor, 0, 0}
with tensor 0 = the initial latent and tensor t = the renoising noise of step t - 1; group g's
four words give elements 4g .. 4g + 3 by the Box-Muller transform with u = (word + 0.5) / 2^32
(the uniforms formed in single precision as on the device, the transform in float64).
"""
from __future__ import annotations

import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = 0x9E3779B9, 0xBB67AE85
MASK = np.uint64(0xFFFFFFFF)

# (counter, key, output) from the generator's published known-answer tests
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int):
    """Vectorised over arrays of counters (uint32 values); returns four uint64 arrays."""
    c = [np.asarray(x, dtype=np.uint64) & MASK for x in (c0, c1, c2, c3)]
    c = [np.broadcast_to(x, np.broadcast(*c).shape).copy() for x in c]
    k0, k1 = int(k0) & 0xFFFFFFFF, int(k1) & 0xFFFFFFFF
    for _ in range(10):
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return c


def normals(seed: int, tensor: int, n: int) -> np.ndarray:
    """The first n (a multiple of 4) N(0, 1) values of noise tensor ``tensor`` (float64)."""
    g = np.arange(n // 4, dtype=np.uint64)
    r = philox4x32_10(g, tensor, 0, 0, seed & 0xFFFFFFFF, seed >> 32)
    out = np.empty((n // 4, 4))
    for p in range(2):
        # the uniforms exactly as the device forms them: the 32-bit word rounded to single
        # precision, + 0.5 and * 2^-32 in single precision; the transforms then in float64
        u1 = ((r[2 * p].astype(np.uint32).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -32))
        u2 = ((r[2 * p + 1].astype(np.uint32).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -32))
        u1, u2 = u1.astype(np.float64), u2.astype(np.float64)
        rad = np.sqrt(-2.0 * np.log(u1))
        out[:, 2 * p] = rad * np.cos(2 * np.pi * u2)
        out[:, 2 * p + 1] = rad * np.sin(2 * np.pi * u2)
    return out.reshape(-1)
