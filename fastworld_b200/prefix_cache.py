"""Exact prefix sharing across requests (same contract as fastworld/prefix_cache.py:35-92).

A request is a path of chunk keys; chunk k depends only on keys 0..k (its noise is seeded by
the path prefix), so requests that share a prefix share those chunks bit for bit.  The cache
is a radix tree over chunk keys; a node holds its chunk's latent and decoded frames and,
every ``every`` chunks, a session checkpoint (runtime state + decoder state).

Duck-typed interfaces:
  runtime:  gen_chunk(path, k) -> latent;  prefill(latent, path, k);  state() -> obj;  load(obj);  [reset()]
  decoder:  decode(latent) -> frames [T, 3, H, W] in [-1, 1];  reset();  state() -> obj;  load(obj)
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
    __slots__ = ("children", "lat", "frames", "ckpt", "depth")

    def __init__(self, depth: int):
        self.children, self.lat, self.frames, self.ckpt, self.depth = {}, None, None, None, depth


class PrefixCache:
    def __init__(self, runtime, decoder, every=2):
        """every: checkpoint period in chunks; None disables sharing."""
        self.rt, self.dec, self.every = runtime, decoder, every
        self.root, self.n_ckpt = Node(-1), 0

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
                    child.ckpt = (self.rt.state(), self.dec.state())
                    self.n_ckpt += 1
                node.children[path[k]] = child
                node = child
            st["done"].append(time.time() - t0)
        st["time"] = time.time() - t0
        return frames, st
