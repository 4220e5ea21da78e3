"""Device chunk preparation (``fw_prep``) against the host path and the CPU generator.

The host path (torch, the reference's own noise stream) stays the default; the device path
(``B200StaticMG(..., device_prep=True)``) writes the same chunk info, action windows and image
condition slice bit for bit, draws its noise from Philox-4x32-10 (checked against the CPU
restatement within one bf16 rounding step), and a chunk run on device-prepared inputs equals,
bit for bit, the same chunk run on host-prepared inputs carrying that noise."""
import numpy as np
import pytest
import torch

from fastworld_b200.config import SMALL
from fastworld_b200.prep import path_seed, synthetic_image
from fastworld_b200.weights import synthetic_state_dict

pytestmark = pytest.mark.gpu

PATH = [("img0", (k, c)) for k, c in zip("wsadqwsad", "uijklujki")]


def sessions():
    from fastworld_b200.static import B200StaticMG
    sd = synthetic_state_dict(SMALL, 0)
    img = synthetic_image(SMALL, 5, 10)
    out = []
    for dev in (False, True):
        S = B200StaticMG(SMALL, sd, device_prep=dev)
        S.add_image("img0", img)
        out.append(S)
    return out


def inputs(S):
    return {n: t.clone() for n, t in (("chunk", S.chunk_info), ("kc", S.kc), ("gm", S.gm), ("cc", S.cc),
                                      ("x_in", S.x_in), *((f"noise{i}", t) for i, t in enumerate(S.noise)))}


def test_windows_condition_and_chunk_info_bitwise():
    H, D = sessions()
    for k in range(8):
        H._prep(PATH, k)
        D._prep(PATH, k)
        torch.cuda.synchronize()
        a, b = inputs(H), inputs(D)
        for n in ("chunk", "kc", "gm", "cc"):
            assert torch.equal(a[n], b[n]), (k, n)
        assert D.device_status()[0] == 0


def test_noise_matches_the_cpu_generator():
    from oracle.prep_oracle import normals
    _, D = sessions()
    for k in (0, 3):
        D._prep(PATH, k)
        torch.cuda.synchronize()
        seed = path_seed(PATH[:k + 1])
        for t, buf in enumerate([D.x_in] + D.noise):
            got = buf.float().cpu().numpy().reshape(-1)
            ref = normals(seed, t, got.size)
            ref_bf = torch.from_numpy(ref).float().bfloat16().float().numpy()
            # equal after bf16 rounding except where the device's single-precision log / sincos
            # land on the other side of a rounding boundary: within one bf16 step (2^-7
            # relative) of the float64 value, or 1e-5 absolute near zero
            err = np.abs(got - ref) - (np.abs(ref) * 2.0 ** -7 + 1e-5)
            i = int(np.argmax(err))
            assert err[i] <= 0, (t, i, float(got[i]), float(ref[i]))
            assert np.mean(got == ref_bf) > 0.995
            assert abs(got.mean()) < 0.02 and abs(got.std() - 1) < 0.02
        assert not torch.equal(D.x_in, D.noise[0])


def test_chunk_on_device_prepared_inputs_equals_host_path():
    H, D = sessions()
    for k in range(3):
        D._prep(PATH, k)
        H._prep(PATH, k)
        H.x_in.copy_(D.x_in)
        for a, b in zip(H.noise, D.noise):
            a.copy_(b)
        H._chunk(k == 0)
        D._chunk(k == 0)
        torch.cuda.synchronize()
        assert torch.equal(H.out, D.out), k
        assert torch.equal(H._blob, D._blob), k
    assert D.device_status()[0] == 0
