"""CUDA-graph capture for static-shape runtimes (same contract as fastworld/graph.py:13-37).

``capture({key: fn}, warmup, save, load)`` snapshots the session state, warms every callable
up on a side stream, records each callable as one ``torch.cuda.CUDAGraph`` (all graphs share
one memory pool, only one runs at a time) and restores the snapshot, so that a later
``replay()`` starts from the state the caller had before capturing.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def capture(fns, warmup: int = 2, save=None, load=None):
    """fns: {key: callable} -> {key: CUDAGraph}."""
    snapshot = save() if save else None
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in fns.values():
            for _ in range(warmup):
                fn()
    torch.cuda.current_stream().wait_stream(side)
    graphs, pool = {}, None
    for key, fn in fns.items():
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            fn()
        pool = g.pool()
        graphs[key] = g
    if load:
        load(snapshot)
    torch.cuda.synchronize()
    return graphs


def state_bytes(tensors) -> int:
    return sum(t.numel() * t.element_size() for t in tensors if torch.is_tensor(t))
