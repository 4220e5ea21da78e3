"""TAEHV decoder, host side (no GPU): the oracle's streaming form, the weight layouts the kernels
assume, the algebra the engine relies on (TGrow before the upsample), and the C-ABI's tensor
table."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from fastworld_b200.vae import TAEHV_SMALL, TAEW2_1, pack_weights, param_specs, synthetic_state_dict
from oracle.taehv_oracle import TaehvOracle, clamp, tgrow


def _lat(cfg, frames, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(16, frames, cfg.lat_h, cfg.lat_w, generator=g)


def test_streaming_equals_whole_sequence():
    """Decoding chunk by chunk with carried MemBlock memory equals decoding every latent frame in
    one call (StreamingTAEHV's contract), including the first-chunk trim."""
    cfg = TAEHV_SMALL
    sd = synthetic_state_dict(cfg, 1)
    lat = _lat(cfg, 3 * cfg.lat_frames, 2)
    whole = TaehvOracle(cfg, sd)
    ref = whole.decode(lat)
    stream = TaehvOracle(cfg, sd)
    parts = [stream.decode(lat[:, i * cfg.lat_frames:(i + 1) * cfg.lat_frames]) for i in range(3)]
    got = torch.cat(parts, 0)
    assert got.shape == ref.shape == (3 * cfg.frames_out - cfg.trim, 3, 8 * cfg.lat_h, 8 * cfg.lat_w)
    assert torch.allclose(got, ref, atol=1e-5, rtol=0)
    assert parts[0].shape[0] == cfg.frames_out - cfg.trim and parts[1].shape[0] == cfg.frames_out


def test_state_restore_reproduces_the_branch():
    cfg = TAEHV_SMALL
    sd = synthetic_state_dict(cfg, 1)
    o = TaehvOracle(cfg, sd)
    o.decode(_lat(cfg, cfg.lat_frames, 3))
    st = o.state()
    a = o.decode(_lat(cfg, cfg.lat_frames, 4))
    o.decode(_lat(cfg, cfg.lat_frames, 5))
    o.load(st)
    b = o.decode(_lat(cfg, cfg.lat_frames, 4))
    assert torch.equal(a, b)


def test_outputs_in_range_and_not_saturated():
    cfg = TAEHV_SMALL
    o = TaehvOracle(cfg, synthetic_state_dict(cfg, 0))
    y = o.decode(_lat(cfg, cfg.lat_frames, 6))
    assert float(y.min()) >= -1 and float(y.max()) <= 1
    inside = ((y > -1) & (y < 1)).float().mean()
    assert 0.5 < float(inside) < 1.0   # the clamp is exercised, most values are not clipped


def test_tgrow_commutes_with_upsample():
    """The engine applies TGrow (a 1 x 1 conv) before the 2x nearest upsample, 4x less work."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 64, 5, 7, generator=g)
    w = torch.randn(128, 64, 1, 1, generator=g)
    a = tgrow(F.interpolate(x, scale_factor=2, mode="nearest"), w, 2)
    b = F.interpolate(tgrow(x, w, 2), scale_factor=2, mode="nearest")
    assert torch.allclose(a, b, atol=1e-5)


def _im2col_conv(x, wk, taps, cin):
    """Conv from the packed [Cout, taps * Cin] layout with K ordered (tap, channel), x NCHW."""
    T, C, H, W = x.shape
    xp = F.pad(x, (1, 1, 1, 1)) if taps == 9 else x
    cols = []
    for p in range(taps):
        dy, dx = (p // 3, p % 3) if taps == 9 else (0, 0)
        cols.append(xp[:, :, dy:dy + H, dx:dx + W])
    a = torch.stack(cols, 1).permute(0, 3, 4, 1, 2).reshape(T * H * W, taps * cin)   # (tap, channel)
    y = a @ wk[:, :taps * cin].float().t()
    return y.reshape(T, H, W, -1).permute(0, 3, 1, 2)


def test_packed_weight_layout():
    cfg = TAEHV_SMALL
    sd = synthetic_state_dict(cfg, 0)
    pk = pack_weights(cfg, sd)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 128, cfg.lat_h, cfg.lat_w, generator=g)
    ref = F.conv2d(x, sd["decoder.3.conv.0.weight"].float(), padding=1)
    got = _im2col_conv(x, pk["mb0.w0"], 9, 128)
    assert torch.allclose(got, ref, atol=1e-3)
    # first conv: 9 taps x 16 latent channels, zero-padded to 192 columns
    x16 = torch.randn(2, 16, cfg.lat_h, cfg.lat_w, generator=g)
    assert pk["conv_in.w"].shape == (64, 192) and torch.all(pk["conv_in.w"][:, 144:] == 0)
    ref = F.conv2d(x16, sd["decoder.1.weight"].float(), padding=1)
    assert torch.allclose(_im2col_conv(x16, pk["conv_in.w"], 9, 16), ref, atol=1e-3)
    # the transposed last conv: row (ky * 3 + kx) * 3 + c
    w22 = sd["decoder.22.weight"]
    assert pk["conv_out.wt"].shape == (32, 64) and torch.all(pk["conv_out.wt"][27:] == 0)
    assert torch.equal(pk["conv_out.wt"][(2 * 3 + 1) * 3 + 2], w22[2, :, 2, 1])
    assert pk["tgrow1.w"].shape == (128, 64)


def test_clamp_is_soft_and_bounded():
    x = torch.tensor([-100.0, -3.0, 0.0, 1.0, 100.0])
    y = clamp(x)
    assert float(y.abs().max()) <= 3 and abs(float(y[3]) - 3 * torch.tanh(torch.tensor(1 / 3)).item()) < 1e-6


def test_taew2_1_shapes():
    """Sizes the reference quotes for TinyVAE: 36 MiB of state (docs/models/mg2.md:62), 12
    frames per chunk of 3 latent frames at 352 x 640, 9 for a stream's first chunk."""
    cfg = TAEW2_1
    assert abs(cfg.state_bytes() / 2 ** 20 - 36.1) < 0.1
    assert cfg.frames_out == 12 and cfg.trim == 3
    assert (8 * cfg.lat_h, 8 * cfg.lat_w) == (352, 640)
    names = [n for n, *_ in param_specs(cfg)]
    assert names[0] == "decoder.1.weight" and names[-1] == "decoder.22.bias"
    assert "decoder.7.conv.weight" in names and "decoder.20.weight" in names and len(names) == 2 + 9 * 6 + 6 + 2


def test_capi_tensor_table():
    from fastworld_b200 import _lib
    from fastworld_b200.vae import make_config
    L = _lib.lib()
    c = make_config(TAEW2_1)
    h = ctypes.c_void_p()
    assert L.fw_taehv_create(ctypes.byref(c), ctypes.byref(h)) == 0
    try:
        infos = {}
        for i in range(L.fw_taehv_tensor_count(h)):
            inf = _lib.FwTensorInfo()
            assert L.fw_taehv_tensor_info_at(h, i, ctypes.byref(inf)) == 0
            infos[inf.name.decode()] = (inf.kind, tuple(inf.shape[j] for j in range(inf.ndim)), inf.bytes)
        assert infos["mem"][2] == TAEW2_1.state_bytes()
        assert infos["lat"][1] == (16, 3, 44, 80) and infos["rgb"][1] == (12, 3, 352, 640)
        assert 1.0e9 < infos["work"][2] < 1.3e9 and infos["work"][0] == _lib.KIND_WORKSPACE
        pk = pack_weights(TAEW2_1, synthetic_state_dict(TAEW2_1, 0))
        weights = {k for k, v in infos.items() if v[0] == _lib.KIND_WEIGHT}
        assert weights == set(pk)
        for k in weights:
            assert tuple(pk[k].shape) == infos[k][1], k
        assert L.fw_taehv_finalize(h) == -5   # nothing bound
        assert L.fw_taehv_bind(h, b"nope", ctypes.c_void_p(16), 16) == -1
    finally:
        L.fw_taehv_destroy(h)
    bad = make_config(TAEW2_1)
    bad.lat_w = 72
    assert L.fw_taehv_create(ctypes.byref(bad), ctypes.byref(h)) == -2
