"""Tensor parallelism on the CPU, no GPU: the sharding rules, the engine's
per-rank tensor table, and the partition of one block over a 2-rank gloo group, which must
reproduce the single-process oracle block."""
import ctypes
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from fastworld_b200.config import SMALL_TP, WAN14B
from fastworld_b200.weights import shard_state_dict, shard_tensor, synthetic_state_dict


def test_shards_concatenate_to_full_tensors():
    cfg = SMALL_TP
    full = synthetic_state_dict(cfg, 0)
    world = 2
    parts = [shard_state_dict(cfg, full, r, world) for r in range(world)]
    for name, t in full.items():
        ps = [p[name] for p in parts]
        if all(torch.equal(x, t) for x in ps):
            continue                                   # replicated
        dim = 1 if name.endswith((".sa.o.w", ".ca.o.w", ".ffn.2.w")) else 0
        assert torch.equal(torch.cat(ps, dim), t), name
    # drawing shards directly gives the same values as sharding the full dict
    direct = synthetic_state_dict(cfg, 0, shard=(1, world))
    assert all(torch.equal(direct[k], parts[1][k]) for k in direct)


def test_rank_tensor_table_matches_packed_shards():
    from fastworld_b200 import _lib
    from fastworld_b200.static import pack_weights
    L = _lib.lib() if os.path.exists(_lib.LIB_PATH) else None
    if L is None:
        from fastworld_b200 import build
        build.build()
        L = _lib.lib()
    cfg = SMALL_TP
    full = synthetic_state_dict(cfg, 0)
    for rank in range(2):
        packed = pack_weights(cfg, shard_state_dict(cfg, full, rank, 2))
        c = _lib.make_config(cfg, 2, rank)
        h = ctypes.c_void_p()
        assert L.fw_create(ctypes.byref(c), ctypes.byref(h)) == 0
        shapes = {}
        for i in range(L.fw_tensor_count(h)):
            inf = _lib.FwTensorInfo()
            assert L.fw_tensor_info_at(h, i, ctypes.byref(inf)) == 0
            shapes[inf.name.decode()] = (inf.kind, tuple(inf.shape[j] for j in range(inf.ndim)))
        w = {k: s for k, (kind, s) in shapes.items() if kind == _lib.KIND_WEIGHT}
        assert set(w) == set(packed)
        for k, s in w.items():
            assert tuple(packed[k].shape) == s, k
        # history: 2 chunk slots x this rank's 2 heads
        assert shapes["hk.0"][1] == (1, 2 * cfg.tokens, 2, 128)
        # a launch before fw_tp_init is refused
        assert L.fw_chunk(h, 1, None) == -7
        L.fw_destroy(h)


def test_tp_config_checks():
    from fastworld_b200 import _lib
    L = _lib.lib()

    def create(cfg, world, rank=0):
        c = _lib.make_config(cfg, world, rank)
        h = ctypes.c_void_p()
        rc = L.fw_create(ctypes.byref(c), ctypes.byref(h))
        if rc == 0:
            L.fw_destroy(h)
        return rc

    assert create(SMALL_TP, 3) == -2                  # 4 heads over 3 ranks
    assert create(SMALL_TP, 2, 2) == -1               # rank out of range
    assert create(SMALL_TP.replace(action_blocks=(0,)), 2) == -2
    assert create(SMALL_TP.replace(hist_chunks=0), 1) == -1
    for world in (1, 2, 4, 8):                        # the 14B shape at every TP size of the box
        assert create(WAN14B, world) == 0
    assert shard_tensor(WAN14B, "b3.ffn.2.w", torch.empty(5120, 13824), 7, 8).shape == (5120, 1728)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _block_rank(rank, world, port, q):
    from oracle.mg2_oracle import Oracle
    from oracle.tp_oracle import block_rank
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(2)
    cfg = SMALL_TP.replace(layers=1, hist_chunks=1)
    full = synthetic_state_dict(cfg, 0)
    W = {k: v.float() for k, v in shard_state_dict(cfg, full, rank, world).items()}
    g = torch.Generator().manual_seed(5)
    xs = torch.randn(cfg.tokens, cfg.dim, generator=g)
    hk = torch.randn(cfg.tokens, cfg.heads, cfg.head_dim, generator=g)
    hv = torch.randn(cfg.tokens, cfg.heads, cfg.head_dim, generator=g)
    vis = torch.randn(cfg.ctx_tokens, cfg.ctx_dim, generator=g)
    orc = Oracle(cfg, full, round_interface=False)
    Hl = cfg.heads // world

    def allreduce(t):
        t = t.clone()
        torch.distributed.all_reduce(t)
        return t

    out = block_rank(orc, W, 0, xs, 750.0, hk[:, rank * Hl:(rank + 1) * Hl], hv[:, rank * Hl:(rank + 1) * Hl], vis,
                     2, allreduce, world)
    ref = orc.block_forward(xs, 750.0, hk, hv, vis, k=2) if rank == 0 else None
    q.put((rank, out, ref))
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_tp_block_partition_matches_oracle_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_block_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r: (o, ref) for r, o, ref in (q.get(timeout=300) for _ in range(2))}
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = res[0][1]
    for r in range(2):
        err = float((res[r][0] - ref).norm() / ref.norm())
        assert err < 1e-5, (r, err)        # fp32 on both sides; only the summation order differs
    assert torch.equal(res[0][0], res[1][0])   # every rank holds the same residual stream
