"""Exact prefix sharing across requests, with the checkpoint pool as part of the tree.

Contract kept from fastworld/prefix_cache.py:35-92: ``PrefixCache(runtime, decoder, every)``;
``serve(path)`` returns one uint8 frame tensor per chunk and a stats dict with ``hit``,
``restored``, ``replayed``, ``generated``, ``done`` (per-chunk completion times) and ``time``;
``n_ckpt`` counts checkpoints taken.  Chunk k of a path depends only on the keys 0..k (its
noise is seeded by that prefix), so a cached prefix is served bit for bit, and a request that
leaves the cached tree resumes from a checkpoint of the session taken on its prefix.

Structure (own design):

* ``Chunk`` nodes form a trie over chunk keys.  Each node knows its parent and depth (its
  chunk index) and stores its latent and frames; a node that holds a checkpoint carries a
  ``Slot``.
* ``CheckpointPool`` owns every slot: the bound on how many are held, least-recently-used
  eviction, recycling of an evicted slot's buffers (``runtime.state_into``), and placement on
  devices.  The anchor of a restore is the nearest ancestor holding a slot, found by following
  parent links up from the deepest matched node; evicting a slot just moves later anchors up.
* Placement: a slot records the device its snapshot lives on.  New checkpoints go to the first
  device in ``devices`` (default: the runtime's own) that holds fewer than ``per_device``
  slots, so a session whose GPU is full spills checkpoints into a peer GPU's HBM
  (``runtime.state(device=...)``, written over NVLink) and restores them with a peer read
  (``runtime.load``); when every device is full the least recently used slot is recycled in
  place.  fastworld keeps every checkpoint on the GPU that made it (README.md:161-162).

Duck-typed interfaces:
  runtime:  gen_chunk(path, k) -> latent;  prefill(latent, path, k);  state() -> obj;  load(obj);
            [reset()];  [state_into(obj) -> obj];  [state(device=d) -> obj on device d]
  decoder:  decode(latent) -> frames [T, 3, H, W] in [-1, 1];  reset();  state() -> obj;  load(obj)
"""
from __future__ import annotations

import itertools
import time
from typing import Dict, Hashable, List, Optional, Sequence

import torch


def to_u8(frames: torch.Tensor) -> torch.Tensor:
    """Frames in [-1, 1] to uint8 [0, 255] on the host (the served format)."""
    return frames.clamp(-1.0, 1.0).add(1.0).mul(127.5).round().to(torch.uint8).cpu()


def _device_sync() -> None:
    if torch.cuda.is_available():
        torch.cuda.synchronize()


FULL = object()   # placement answer: no device has room, recycle a slot


class Slot:
    """A held checkpoint: runtime and decoder snapshots, where they live, when last used."""

    __slots__ = ("runtime_state", "decoder_state", "device", "stamp")

    def __init__(self, runtime_state, decoder_state, device, stamp: int):
        self.runtime_state, self.decoder_state = runtime_state, decoder_state
        self.device, self.stamp = device, stamp


class Chunk:
    """Trie node for chunk ``depth`` of every path through it."""

    __slots__ = ("key", "parent", "depth", "kids", "lat", "frames", "slot")

    def __init__(self, key: Hashable = None, parent: Optional["Chunk"] = None):
        self.key, self.parent = key, parent
        self.depth = parent.depth + 1 if parent is not None else -1
        self.kids: Dict[Hashable, Chunk] = {}
        self.lat = self.frames = self.slot = None

    def lineage(self, stop: Optional["Chunk"] = None) -> List["Chunk"]:
        """Nodes from just below ``stop`` (default: the root) down to this one, in chunk order."""
        out, n = [], self
        while n is not stop and n.parent is not None:
            out.append(n)
            n = n.parent
        out.reverse()
        return out


def _device_of(state) -> Optional[torch.device]:
    blob = getattr(state, "blob", None)
    if isinstance(blob, torch.Tensor):
        return blob.device
    if isinstance(getattr(state, "device", None), torch.device):
        return state.device
    if isinstance(state, torch.Tensor):
        return state.device
    if isinstance(state, (list, tuple)) and state and isinstance(state[0], torch.Tensor):
        return state[0].device
    return None


class CheckpointPool:
    """Checkpoints held by tree nodes: bound, LRU eviction, buffer recycling, device placement."""

    def __init__(self, runtime, decoder, capacity: Optional[int] = None, devices: Optional[Sequence] = None,
                 per_device: Optional[int] = None):
        self.rt, self.dec = runtime, decoder
        self.capacity = capacity
        # None = wherever the runtime puts its snapshots
        self.devices = [torch.device(d) if isinstance(d, (str, int)) else d for d in devices] if devices else [None]
        self.per_device = per_device
        self.holders: List[Chunk] = []
        self.made = self.evicted = 0
        self._stamps = itertools.count(1)

    def anchor(self, node: Chunk) -> Optional[Chunk]:
        """Deepest node on ``node``'s root path (itself included) that holds a checkpoint."""
        while node is not None and node.slot is None:
            node = node.parent
        return node

    def _count_on(self, dev) -> int:
        return sum(1 for n in self.holders if n.slot.device == dev or dev is None)

    def _place(self):
        """A device with room for one more checkpoint, or FULL when the pool is full."""
        if self.capacity is not None and len(self.holders) >= self.capacity:
            return FULL
        for dev in self.devices:
            if self.per_device is None or self._count_on(dev) < self.per_device:
                return dev
        return FULL

    def _snapshot(self, dev):
        if dev is None or _device_of_rt(self.rt) == dev:
            return self.rt.state()
        return self.rt.state(device=dev)

    def take(self, node: Chunk) -> None:
        """Checkpoint the session (positioned just after ``node``'s chunk) into ``node``."""
        where = self._place()
        if where is not FULL:
            rt_state = self._snapshot(where)
        else:   # full: recycle the least recently used slot in place
            victim = min(self.holders, key=lambda n: n.slot.stamp)
            old, victim.slot = victim.slot, None
            self.holders.remove(victim)
            self.evicted += 1
            recycle = getattr(self.rt, "state_into", None)
            rt_state = recycle(old.runtime_state) if recycle is not None else self._snapshot(old.device)
        node.slot = Slot(rt_state, self.dec.state(), _device_of(rt_state), next(self._stamps))
        self.holders.append(node)
        self.made += 1

    def restore(self, node: Chunk) -> None:
        slot = node.slot
        slot.stamp = next(self._stamps)
        self.rt.load(slot.runtime_state)
        self.dec.load(slot.decoder_state)

    def bytes_by_device(self) -> Dict[str, int]:
        out: Dict[str, int] = {}
        for n in self.holders:
            blob = getattr(n.slot.runtime_state, "blob", None)
            nb = blob.numel() * blob.element_size() if isinstance(blob, torch.Tensor) else 0
            key = str(n.slot.device)
            out[key] = out.get(key, 0) + nb
        return out


def _device_of_rt(rt):
    dev = getattr(rt, "dev", None)
    return dev if isinstance(dev, torch.device) else None


class PrefixCache:
    def __init__(self, runtime, decoder, every: Optional[int] = 2, max_checkpoints: Optional[int] = None,
                 devices: Optional[Sequence] = None, per_device: Optional[int] = None):
        """every: checkpoint period in chunks (None: no sharing, every request from scratch).
        max_checkpoints: most checkpoints held at once (None: unbounded).  devices / per_device:
        checkpoint placement (default: all on the runtime's device)."""
        self.rt, self.dec, self.every = runtime, decoder, every
        self.root = Chunk()
        self.pool = CheckpointPool(runtime, decoder, max_checkpoints, devices, per_device)

    # counters kept under the reference's names
    @property
    def n_ckpt(self) -> int:
        return self.pool.made

    @property
    def n_evicted(self) -> int:
        return self.pool.evicted

    @property
    def _held(self) -> List[Chunk]:
        return self.pool.holders

    def _deepest_match(self, path: Sequence) -> Chunk:
        node = self.root
        if self.every:
            for key in path:
                kid = node.kids.get(key)
                if kid is None:
                    break
                node = kid
        return node

    def _position_after(self, node: Chunk, path: Sequence, stats: dict) -> None:
        """Bring the runtime and decoder to the state just after ``node``'s chunk."""
        anchor = self.pool.anchor(node)
        if anchor is None:
            if hasattr(self.rt, "reset"):
                self.rt.reset()
            self.dec.reset()
        else:
            self.pool.restore(anchor)
            stats["restored"] = 1
        for c in node.lineage(stop=anchor):     # chunks after the anchor, from their latents
            self.rt.prefill(c.lat, path, c.depth)
            self.dec.decode(c.lat)
            stats["replayed"] += 1

    @torch.no_grad()
    def serve(self, path: Sequence):
        """Frames for every chunk of ``path`` (uint8, host) and the stats of this request."""
        _device_sync()
        start = time.time()
        node = self._deepest_match(path)
        cached = node.lineage()
        frames = [c.frames for c in cached]
        stats = {"hit": len(cached), "restored": 0, "replayed": 0, "generated": len(path) - len(cached), "done": []}
        if len(cached) < len(path):
            self._position_after(node, path, stats)
        _device_sync()
        stats["done"] = [time.time() - start] * len(cached)
        last = len(path) - 1
        for k in range(len(cached), len(path)):
            lat = self.rt.gen_chunk(path, k)
            fr = to_u8(self.dec.decode(lat))
            frames.append(fr)
            if self.every:
                node = node.kids.setdefault(path[k], Chunk(path[k], node))
                node.lat, node.frames = lat.clone(), fr
                # a checkpoint closes every `every`-th chunk, except the request's last one
                if k < last and k % self.every == self.every - 1:
                    self.pool.take(node)
            stats["done"].append(time.time() - start)
        stats["time"] = time.time() - start
        return frames, stats
