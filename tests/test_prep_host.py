"""Device chunk preparation, host side: the counter-based generator against its published
known-answer vectors (through the library's host entry point and the CPU restatement), and the
action chunks the host hands to ``fw_prep`` cover every window position of prep.action_windows
(the restatement of static.py:85-112)."""
import ctypes

import pytest

from fastworld_b200.config import MG2, SMALL
from fastworld_b200.prep import KEYS, CAM, action_windows, chunk_of_pixel_frame, device_prep_actions, window_chunks
from oracle.prep_oracle import PHILOX_KAT, philox4x32_10


def test_philox_known_answers_library_and_oracle():
    from fastworld_b200 import _lib
    L = _lib.lib()
    for ctr, key, want in PHILOX_KAT:
        C, K, O = (ctypes.c_uint * 4)(*ctr), (ctypes.c_uint * 2)(*key), (ctypes.c_uint * 4)()
        assert L.fw_philox4x32_10(C, K, O) == 0
        assert tuple(O) == want
        got = philox4x32_10(*ctr, *key)
        assert tuple(int(x) for x in got) == want


@pytest.mark.parametrize("cfg", [MG2, SMALL])
def test_window_chunks_cover_the_window(cfg):
    r, F, pad = cfg.time_ratio, cfg.frames, cfg.pad_t
    for k in range(24):
        lo, hi = window_chunks(cfg, k)
        assert hi == k and hi - lo + 1 <= 4
        for i in range(cfg.kc_len):
            q = r * F * k + i - pad
            j = 0 if q < 0 else chunk_of_pixel_frame(q, F, r)
            assert lo <= j <= hi


def test_device_prep_actions_reproduce_the_host_windows():
    """Gathering from (j_lo, per-chunk vectors) with the device kernel's rule gives the host
    windows exactly."""
    import torch
    cfg = MG2
    keys, cams = list(KEYS), list(CAM)
    path = [("img", (keys[i % 5], cams[(3 * i) % 5])) for i in range(12)]
    r, F, pad = cfg.time_ratio, cfg.frames, cfg.pad_t
    for k in range(12):
        kc, gm = action_windows(cfg, path, k)
        lo, acts = device_prep_actions(cfg, path, k)
        rows = []
        for i in range(cfg.kc_len):
            q = r * F * k + i - pad
            j = 0 if q < 0 else chunk_of_pixel_frame(q, F, r)
            rows.append(acts[j - lo])
        dev = torch.tensor(rows, dtype=torch.float32).bfloat16()
        assert torch.equal(dev[:, :4], kc)
        assert torch.equal(torch.stack([dev[r * f:r * f + pad, 4:6] for f in range(F)]), gm)
