"""fastworld_b200: the Matrix-Game-2-shaped causal Wan DiT chunk forward on B200 (sm_100a).

Drop-in for the hot path of fastworld (``StaticMG`` + ``graph.capture`` + ``PrefixCache``):
``B200StaticMG`` keeps the session API, and its chunk runs hand-written tcgen05/TMA kernels
through the C ABI in ``include/fastworld_b200.h``.
"""
from .config import BLOCK, MG2, PRESETS, SMALL, TINY, WAN14B, DiTConfig
from .graph import capture, state_bytes
from .prefix_cache import PrefixCache, to_u8
from .prep import CAM, KEYS, action_windows, draw_noise, path_seed, synthetic_image

__all__ = ["BLOCK", "CAM", "KEYS", "MG2", "PRESETS", "SMALL", "TINY", "WAN14B", "DiTConfig", "PrefixCache",
           "B200StaticMG", "action_windows", "capture", "draw_noise", "path_seed", "state_bytes",
           "synthetic_image", "to_u8"]


def __getattr__(name):
    if name == "B200StaticMG":
        from .static import B200StaticMG
        return B200StaticMG
    raise AttributeError(name)
