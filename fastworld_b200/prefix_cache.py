"""Exact prefix sharing across requests (same contract as fastworld/prefix_cache.py:35-92).

A request is a path of chunk keys; chunk k depends only on keys 0..k (its noise is seeded by
the path prefix), so requests that share a prefix share those chunks bit for bit.  The cache
is a radix tree over chunk keys; a node holds its chunk's latent and decoded frames and,
every ``every`` chunks, a session checkpoint (runtime state + decoder state).

Duck-typed interfaces:
  runtime:  gen_chunk(path, k) -> latent;  prefill(latent, path, k);  state() -> obj;  load(obj);  [reset()]
            [state_into(obj) -> obj: snapshot into an existing checkpoint's buffers]
  decoder:  decode(latent) -> frames [T, 3, H, W] in [-1, 1];  reset();  state() -> obj;  load(obj)

Beyond the reference (which keeps every checkpoint, README.md:161-162): ``max_checkpoints``
bounds the checkpoints held at once.  When a new checkpoint would exceed it, the least
recently used one (created or restored longest ago) is evicted: its node keeps its latent and
frames, so later requests through it still hit, and a restore falls back to the nearest
earlier checkpoint (or a fresh session) and replays the chunks after it, so results do not
change.  With a runtime that offers ``state_into``, the evicted checkpoint's device buffers
are reused for the new one (a fixed pool of session-state buffers: no allocation once the
pool is full).
"""
from __future__ import annotations

import time

import torch


def to_u8(frames: torch.Tensor) -> torch.Tensor:
    return ((frames.clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).cpu()


def _sync():
    if torch.cuda.is_available():
        torch.cuda.synchronize()


class Node:
    __slots__ = ("children", "lat", "frames", "ckpt", "depth", "last_use")

    def __init__(self, depth: int):
        self.children, self.lat, self.frames, self.ckpt, self.depth = {}, None, None, None, depth
        self.last_use = 0


class PrefixCache:
    def __init__(self, runtime, decoder, every=2, max_checkpoints=None):
        """every: checkpoint period in chunks; None disables sharing.  max_checkpoints: at most
        this many checkpoints held at once (least recently used evicted); None = unbounded."""
        self.rt, self.dec, self.every = runtime, decoder, every
        self.root, self.n_ckpt = Node(-1), 0
        self.max_ckpt, self.n_evicted, self._clock = max_checkpoints, 0, 0
        self._held = []   # nodes holding a checkpoint

    def _tick(self, node):
        self._clock += 1
        node.last_use = self._clock

    def _checkpoint(self, node):
        """Snapshot the session into `node`, evicting the least recently used checkpoint first
        when the bound is reached (its buffers are reused when the runtime can write into them)."""
        reuse = None
        if self.max_ckpt is not None and len(self._held) >= self.max_ckpt:
            victim = min(self._held, key=lambda n: n.last_use)
            self._held.remove(victim)
            reuse, victim.ckpt = victim.ckpt, None
            self.n_evicted += 1
        if reuse is not None and hasattr(self.rt, "state_into"):
            rt_state = self.rt.state_into(reuse[0])
        else:
            rt_state = self.rt.state()
        node.ckpt = (rt_state, self.dec.state())
        self._held.append(node)
        self._tick(node)
        self.n_ckpt += 1

    def _fresh(self):
        if hasattr(self.rt, "reset"):
            self.rt.reset()
        self.dec.reset()

    @torch.no_grad()
    def serve(self, path):
        """Returns (list of uint8 frame tensors, one per chunk; stats dict)."""
        _sync()
        t0 = time.time()
        n = len(path)
        node, chain = self.root, []
        if self.every:
            for key in path:
                nxt = node.children.get(key)
                if nxt is None:
                    break
                node = nxt
                chain.append(node)
        m = len(chain)
        st = dict(hit=m, restored=0, replayed=0, generated=n - m, done=[])
        frames = [c.frames for c in chain]
        if m < n:
            ck = max((i for i, c in enumerate(chain) if c.ckpt is not None), default=-1)
            if ck >= 0:
                self._tick(chain[ck])
                rt_state, dec_state = chain[ck].ckpt
                self.rt.load(rt_state)
                self.dec.load(dec_state)
                st["restored"] = 1
            else:
                self._fresh()
            for k in range(ck + 1, m):      # replay the matched chunks after the checkpoint
                self.rt.prefill(chain[k].lat, path, k)
                self.dec.decode(chain[k].lat)
                st["replayed"] += 1
        _sync()
        st["done"] = [time.time() - t0] * m
        node = chain[-1] if chain else self.root
        for k in range(m, n):
            lat = self.rt.gen_chunk(path, k)
            fr = to_u8(self.dec.decode(lat))
            frames.append(fr)
            if self.every:
                child = Node(k)
                child.lat, child.frames = lat.clone(), fr
                if (k + 1) % self.every == 0 and k < n - 1:
                    self._checkpoint(child)
                node.children[path[k]] = child
                node = child
            st["done"].append(time.time() - t0)
        st["time"] = time.time() - t0
        return frames, st
