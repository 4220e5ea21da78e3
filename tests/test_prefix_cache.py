"""PrefixCache semantics (fastworld/prefix_cache.py:47-92) with a deterministic fake runtime:
sharing, checkpoint restore and replay must reproduce generating every request from scratch."""
import hashlib

import torch

from fastworld_b200.prefix_cache import PrefixCache


class FakeRuntime:
    """State = running hash of the chunks advanced; a chunk's latent depends on the state and key."""

    def __init__(self):
        self.h = b""
        self.calls = {"gen": 0, "prefill": 0, "load": 0}

    def _adv(self, key):
        self.h = hashlib.sha1(self.h + repr(key).encode()).digest()

    def gen_chunk(self, path, k):
        self.calls["gen"] += 1
        self._adv(path[k])
        return torch.tensor(list(self.h[:8]), dtype=torch.float32)

    def prefill(self, lat, path, k):
        self.calls["prefill"] += 1
        self._adv(path[k])

    def state(self):
        return self.h

    def load(self, st):
        self.calls["load"] += 1
        self.h = st

    def reset(self):
        self.h = b""


class FakeDecoder:
    def __init__(self):
        self.n = 0

    def decode(self, lat):
        return (lat / 255.0)[None, None, None, :].expand(1, 3, 1, 8) * 2 - 1

    def reset(self):
        pass

    def state(self):
        return None

    def load(self, st):
        pass


def test_sharing_matches_scratch():
    paths = [[("img", a) for a in p] for p in (
        "wwww", "wwss", "wwsa", "wadd", "wwww", "ww", "wwsaq")]
    ref_rt = FakeRuntime()
    scratch = PrefixCache(ref_rt, FakeDecoder(), every=None)
    rt = FakeRuntime()
    cache = PrefixCache(rt, FakeDecoder(), every=2)
    for p in paths:
        a, _ = scratch.serve(p)
        b, st = cache.serve(p)
        assert len(a) == len(b) == len(p)
        assert all(torch.equal(x, y) for x, y in zip(a, b))
    assert rt.calls["gen"] < ref_rt.calls["gen"]
    assert rt.calls["load"] > 0 and cache.n_ckpt > 0


def test_stats_of_a_rewind():
    rt = FakeRuntime()
    cache = PrefixCache(rt, FakeDecoder(), every=2)
    main = [("img", c) for c in "wwwwwwww"]
    cache.serve(main)
    _, st = cache.serve(main[:5] + [("img", "a")] * 3)
    assert st["hit"] == 5 and st["restored"] == 1 and st["replayed"] == 1 and st["generated"] == 3


class PoolRuntime(FakeRuntime):
    """FakeRuntime whose snapshots are mutable boxes, recycled through state_into."""

    def __init__(self):
        super().__init__()
        self.allocated = 0

    def state(self):
        self.allocated += 1
        return [self.h]

    def state_into(self, box):
        box[0] = self.h
        return box

    def load(self, st):
        self.calls["load"] += 1
        self.h = st[0]


def test_bounded_checkpoints_match_scratch_and_recycle():
    import random
    rng = random.Random(3)
    keys = "wasdq"
    paths = []
    for _ in range(40):   # random prefixes of a few trunks, like rewinds in an explore workload
        trunk = [("img", c) for c in rng.choice(["wwwwwwww", "wwssaadd", "wadqwadq"])]
        cut = rng.randrange(1, 8)
        paths.append(trunk[:cut] + [("img", rng.choice(keys)) for _ in range(rng.randrange(1, 4))])
    scratch = PrefixCache(FakeRuntime(), FakeDecoder(), every=None)
    rt = PoolRuntime()
    cache = PrefixCache(rt, FakeDecoder(), every=2, max_checkpoints=3)
    for p in paths:
        a, _ = scratch.serve(p)
        b, st = cache.serve(p)
        assert all(torch.equal(x, y) for x, y in zip(a, b)), p
    assert len(cache._held) <= 3 and cache.n_evicted > 0
    assert rt.allocated == 3          # the pool never grew past its bound
    assert rt.calls["load"] > 0


class PlacedState:
    def __init__(self, h, device):
        self.h, self.device = h, device


class PlacingRuntime(FakeRuntime):
    """FakeRuntime whose snapshots record the device they were placed on (labels only; nothing
    is allocated on a GPU)."""

    dev = torch.device("cuda:0")

    def __init__(self):
        super().__init__()
        self.placed = []

    def state(self, device=None):
        d = torch.device(device) if device is not None else self.dev
        self.placed.append(d)
        return PlacedState(self.h, d)

    def state_into(self, box):
        box.h = self.h
        return box

    def load(self, st):
        self.calls["load"] += 1
        self.h = st.h


def test_checkpoints_spill_to_a_peer_device_then_recycle():
    main = [("img", c) for c in "wwwwwwwwwwww"]       # 12 chunks: checkpoints after chunks 1, 3, 5, 7, 9
    rt = PlacingRuntime()
    cache = PrefixCache(rt, FakeDecoder(), every=2, devices=["cuda:0", "cuda:1"], per_device=2)
    scratch = PrefixCache(FakeRuntime(), FakeDecoder(), every=None)
    a, _ = scratch.serve(main)
    b, _ = cache.serve(main)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    # two on the session's own GPU, two spilled to the peer, the fifth recycles the oldest in place
    assert [d.index for d in rt.placed] == [0, 0, 1, 1]
    assert cache.n_ckpt == 5 and cache.n_evicted == 1 and len(cache._held) == 4
    devs = sorted(n.slot.device.index for n in cache._held)
    assert devs == [0, 0, 1, 1]
    # a rewind to chunk 6 restores the deepest held checkpoint at or before it (after chunk 5, on the peer)
    c, st = cache.serve(main[:7] + [("img", "a")])
    d, _ = scratch.serve(main[:7] + [("img", "a")])
    assert all(torch.equal(x, y) for x, y in zip(c, d))
    assert st["restored"] == 1 and st["replayed"] == 1
