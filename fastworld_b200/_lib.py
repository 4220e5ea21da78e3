"""ctypes binding of ``libfastworld_b200.so`` (declared in ``include/fastworld_b200.h``).

The library is built in-tree by ``python -m fastworld_b200.build``; importing the binding
never falls back to anything else: a missing library raises immediately.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfastworld_b200.so")

FW_MAX_ACTION_BLOCKS = 64
FW_MAX_STEPS = 16
KIND_WEIGHT, KIND_STATE, KIND_INPUT, KIND_OUTPUT, KIND_WORKSPACE, KIND_STATUS, KIND_DERIVED = range(7)
DT_BF16, DT_F32, DT_I32, DT_U8, DT_F16 = range(5)
EPI_BF16, EPI_GELU_BF16, EPI_RESID_F32, EPI_F32, EPI_GELU_ERF_BF16 = range(5)


class FwConfig(ctypes.Structure):
    _fields_ = [
        ("dim", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
        ("layers", ctypes.c_int), ("freq_dim", ctypes.c_int),
        ("lat_ch", ctypes.c_int), ("cond_ch", ctypes.c_int), ("frames", ctypes.c_int), ("lat_h", ctypes.c_int),
        ("lat_w", ctypes.c_int),
        ("ctx_tokens", ctypes.c_int), ("ctx_dim", ctypes.c_int),
        ("n_action", ctypes.c_int), ("action_blocks", ctypes.c_int * FW_MAX_ACTION_BLOCKS),
        ("act_heads", ctypes.c_int), ("act_head_dim", ctypes.c_int), ("mouse_hidden", ctypes.c_int),
        ("keyboard_hidden", ctypes.c_int), ("mouse_dim", ctypes.c_int), ("keyboard_dim", ctypes.c_int),
        ("time_ratio", ctypes.c_int), ("window", ctypes.c_int),
        ("n_steps", ctypes.c_int), ("steps", ctypes.c_float * FW_MAX_STEPS),
        ("eps", ctypes.c_float), ("eps_ln", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("linear_fp8", ctypes.c_int),
        ("hist_chunks", ctypes.c_int), ("tp_size", ctypes.c_int), ("tp_rank", ctypes.c_int),
    ]


class FwTensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("kind", ctypes.c_int), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_int64 * 5), ("bytes", ctypes.c_size_t)]


FW_PREP_MAX_ACT = 4


class FwPrepArgs(ctypes.Structure):
    _fields_ = [("chunk", ctypes.c_int), ("seed", ctypes.c_ulonglong), ("draw_noise", ctypes.c_int),
                ("cond", ctypes.c_void_p), ("cond_frames", ctypes.c_int), ("j_lo", ctypes.c_int),
                ("n_act", ctypes.c_int), ("actions", ctypes.c_float * (FW_PREP_MAX_ACT * 8))]


class FwTaehvConfig(ctypes.Structure):
    _fields_ = [("lat_ch", ctypes.c_int), ("lat_frames", ctypes.c_int), ("lat_h", ctypes.c_int),
                ("lat_w", ctypes.c_int), ("channels", ctypes.c_int * 4), ("time_up", ctypes.c_int * 3)]


class FwLbConfig(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
                ("layers", ctypes.c_int), ("freq_dim", ctypes.c_int), ("text_len", ctypes.c_int),
                ("text_dim", ctypes.c_int), ("lat_ch", ctypes.c_int), ("y_ch", ctypes.c_int), ("cam_ch", ctypes.c_int),
                ("chunk", ctypes.c_int), ("lat_h", ctypes.c_int), ("lat_w", ctypes.c_int), ("kv_frames", ctypes.c_int),
                ("sink_frames", ctypes.c_int), ("n_steps", ctypes.c_int), ("eps", ctypes.c_float),
                ("timesteps", ctypes.c_float * 8), ("sig_x0", ctypes.c_double * 8), ("an_alpha", ctypes.c_float * 8),
                ("an_sigma", ctypes.c_float * 8)]


_SIGS = {
    "fw_abi_version": (ctypes.c_int, []),
    "fw_launch_count": (ctypes.c_ulonglong, []),
    "fw_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "fw_create": (ctypes.c_int, [ctypes.POINTER(FwConfig), ctypes.POINTER(ctypes.c_void_p)]),
    "fw_tensor_count": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_tensor_info_at": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(FwTensorInfo)]),
    "fw_bind": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t]),
    "fw_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_chunk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "fw_prefill": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "fw_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "fw_destroy": (None, [ctypes.c_void_p]),
    "fw_tap_bytes": (ctypes.c_size_t, [ctypes.c_void_p]),
    "fw_prep": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(FwPrepArgs), ctypes.c_void_p]),
    "fw_philox4x32_10": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint),
                                        ctypes.POINTER(ctypes.c_uint)]),
    "fw_set_tap": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]),
    "fw_copy": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "fw_gemm_bf16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "fw_gemm_e4m3": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_void_p]),
    "fw_quant_e4m3": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_void_p]),
    "fw_ipc_get_handle": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_size_t)]),
    "fw_ipc_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "fw_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_linear_e4m3_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p]),
    "fw_gemm_bf16_resid": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_void_p]),
    "fw_tp_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "fw_tp_init": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p]),
    "fw_tp_peers": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]),
    "fw_tp_reduce_once": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "fw_tp_allreduce": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_void_p]),
    "fw_graph_begin": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_graph_end": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "fw_lb_create": (ctypes.c_int, [ctypes.POINTER(FwLbConfig), ctypes.POINTER(ctypes.c_void_p)]),
    "fw_lb_tensor_count": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_lb_tensor_info_at": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(FwTensorInfo)]),
    "fw_lb_bind": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t]),
    "fw_lb_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_lb_set_prompt": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "fw_lb_chunk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "fw_lb_roll_pieces": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_lb_destroy": (None, [ctypes.c_void_p]),
    "fw_taehv_create": (ctypes.c_int, [ctypes.POINTER(FwTaehvConfig), ctypes.POINTER(ctypes.c_void_p)]),
    "fw_taehv_tensor_count": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_taehv_tensor_info_at": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(FwTensorInfo)]),
    "fw_taehv_bind": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t]),
    "fw_taehv_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "fw_taehv_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "fw_taehv_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "fw_taehv_destroy": (None, [ctypes.c_void_p]),
    "fw_graph_launch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "fw_graph_nodes": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "fw_graph_destroy": (None, [ctypes.c_void_p]),
    "fw_peer_access": (ctypes.c_int, [ctypes.c_int]),
    "fw_selftest_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "fw_selftest_wait": (ctypes.c_int, [ctypes.c_int, ctypes.c_ulonglong, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_void_p, ctypes.c_void_p]),
    "fw_layernorm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p]),
    "fw_rms_rope": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "fw_attention": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
}

_LIB = None


def lib() -> ctypes.CDLL:
    """Load the engine library (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m fastworld_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _LIB = L
    return _LIB


def strerror(rc: int) -> str:
    return lib().fw_strerror(rc).decode()


def check(rc: int, what: str = "call") -> None:
    if rc != 0:
        raise RuntimeError(f"fastworld_b200 {what} failed: {strerror(rc)} (code {rc})")


def make_config(cfg, tp_size: int = 1, tp_rank: int = 0) -> FwConfig:
    """fw_config from a :class:`fastworld_b200.config.DiTConfig` (and this rank's tensor-parallel
    position)."""
    c = FwConfig()
    for f in ("dim", "heads", "head_dim", "ffn", "layers", "freq_dim", "lat_ch", "cond_ch", "frames", "lat_h",
              "lat_w", "ctx_tokens", "ctx_dim", "act_heads", "act_head_dim", "mouse_hidden", "keyboard_hidden",
              "mouse_dim", "keyboard_dim", "time_ratio", "window"):
        setattr(c, f, int(getattr(cfg, f)))
    if len(cfg.action_blocks) > FW_MAX_ACTION_BLOCKS or len(cfg.steps) > FW_MAX_STEPS:
        raise ValueError("too many action blocks or steps")
    c.n_action = len(cfg.action_blocks)
    for i, b in enumerate(cfg.action_blocks):
        c.action_blocks[i] = int(b)
    c.n_steps = len(cfg.steps)
    for i, t in enumerate(cfg.steps):
        c.steps[i] = float(t)
    c.eps, c.eps_ln, c.rope_theta = float(cfg.eps), 1e-5, float(cfg.rope_theta)
    modes = {"bf16": 0, "fp8": 1, "fp8_ffn": 2}
    if cfg.linear not in modes:
        raise ValueError(f"linear dtype {cfg.linear!r}")
    c.linear_fp8 = modes[cfg.linear]
    c.hist_chunks = int(cfg.hist_chunks)
    c.tp_size, c.tp_rank = int(tp_size), int(tp_rank)
    return c


def ptr(t) -> int:
    return t.data_ptr() if t is not None else 0


def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)
