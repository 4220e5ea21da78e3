"""Host logic of the multi-GPU explore workload on the CPU: seeded paths,
rewinds that branch right after a checkpoint, the session partition over ranks, and the
IPC-offer exchange of the cross-GPU phase over a 2-rank gloo process group."""
import os
import socket

import torch
import torch.multiprocessing as mp

from fastworld_b200.explore import make_paths, rewinds, sessions_of


def test_paths_and_rewinds():
    p = make_paths(64, 16, seed=1)
    assert p == make_paths(64, 16, seed=1) and len(p) == 64 and all(len(x) == 16 for x in p)
    assert p != make_paths(64, 16, seed=2)
    for i in range(8):
        for r in rewinds(p[i], 6, 2, seed=i):
            t = len(r) - 2
            assert t % 2 == 0 and 2 <= t < 16 and r[:t] == p[i][:t]


def test_partition_covers_each_session_once():
    for world in (1, 2, 4, 8):
        seen = sorted(i for r in range(world) for i in sessions_of(r, world, 64))
        assert seen == list(range(64))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    offers = [(i, ("handle", rank, i)) for i in sessions_of(rank, world, 8)[:2]]
    got = [None] * world
    torch.distributed.all_gather_object(got, offers)
    # each rank restores checkpoints owned by the next rank
    q.put((rank, [i for i, _ in got[(rank + 1) % world]], [d[1] for _, d in got[(rank + 1) % world]]))
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_offer_exchange_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (s, o)) for r, s, o in (q.get(timeout=120) for _ in range(2)))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == ([1, 3], [1, 1]) and res[1] == ([0, 2], [0, 0])
