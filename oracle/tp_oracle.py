"""Tensor-parallel restatement of one DiT block on the CPU.  TEST INFRASTRUCTURE ONLY.

Only ``tests/`` import this module.  It states, for one rank of a tensor-parallel group, the
computation the engine performs with ``tp_size > 1`` (heads and FFN
columns sharded, NCCL all-reduce after the row-parallel linears), with the all-reduces done
by a caller-supplied ``allreduce(t) -> t`` (a gloo process group in the tests, or a plain
sum over emulated ranks).  Summed over the group it must reproduce
:meth:`oracle.mg2_oracle.Oracle.block` with the full weights, which pins the sharding rules
of ``fastworld_b200.weights.shard_tensor`` and the placement of every collective:

* q/k/v (self and cross) are column-parallel: this rank's heads.  Their RMSNorms run over
  the full hidden width (static.py:208-209, 189-190), so the per-token sums of squares of
  the shards are all-reduced before normalising.
* sa.o, ca.o and ffn.2 are row-parallel: each rank multiplies its input columns; the partial
  outputs are all-reduced, then the bias and the gated residual are applied once.
* ffn.0 is column-parallel (this rank's hidden columns; GELU is elementwise).
* LayerNorms, adaLN modulation, RoPE tables and the residual stream are replicated.
"""
from __future__ import annotations

from typing import Callable, Dict

import torch

from .mg2_oracle import Oracle, attention, apply_rope, gelu_tanh, layer_norm, rope_table


def _lin(W: Dict[str, torch.Tensor], x: torch.Tensor, name: str, bias: bool = True) -> torch.Tensor:
    y = torch.matmul(x, W[f"{name}.w"].t())
    return y + W[f"{name}.b"] if bias else y


def _rms_sharded(x: torch.Tensor, w: torch.Tensor, dim: int, eps: float, allreduce) -> torch.Tensor:
    """RMSNorm over the full width `dim` of a column shard x [M, dim / tp]."""
    ss = allreduce(x.pow(2).sum(-1, keepdim=True))
    return x * torch.rsqrt(ss / dim + eps) * w


def block_rank(orc: Oracle, W: Dict[str, torch.Tensor], i: int, xs: torch.Tensor, t: float, hist_k: torch.Tensor,
               hist_v: torch.Tensor, vis: torch.Tensor, k: int, allreduce: Callable[[torch.Tensor], torch.Tensor],
               tp: int) -> torch.Tensor:
    """One steady block on one rank: xs [L, dim] replicated -> new xs (replicated).

    ``W``: this rank's shard of the flat state dict (fp32); ``hist_k/hist_v``: this rank's
    heads of the history [L_hist, heads / tp, head_dim]."""
    c, p = orc.cfg, f"b{i}"
    F, S, D, HD = c.frames, c.tok_per_frame, c.dim, c.head_dim
    Hl = c.heads // tp
    _, e0 = orc.time_embed(t)
    ee = (W[f"{p}.mod"] + e0).unbind(0)                                      # 6 x [dim], every frame

    def modulate(x, shift, scale):
        return layer_norm(x, eps=c.eps) * (1 + scale) + shift

    fi = rope_table(c, k, orc.freqs)
    # self-attention over this rank's heads
    y = modulate(xs, ee[0], ee[1])
    q = _rms_sharded(_lin(W, y, f"{p}.sa.q"), W[f"{p}.sa.nq.w"], D, c.eps, allreduce).view(-1, Hl, HD)
    kk = _rms_sharded(_lin(W, y, f"{p}.sa.k"), W[f"{p}.sa.nk.w"], D, c.eps, allreduce).view(-1, Hl, HD)
    v = _lin(W, y, f"{p}.sa.v").view(-1, Hl, HD)
    q, kk = apply_rope(q, fi), apply_rope(kk, fi)
    a = attention(q, torch.cat([hist_k, kk], 0), torch.cat([hist_v, v], 0)).reshape(-1, Hl * HD)
    o = allreduce(_lin(W, a, f"{p}.sa.o", bias=False)) + W[f"{p}.sa.o.b"]
    xs = xs + o * ee[2]
    # cross-attention (context K/V of this rank's heads)
    ctx = orc.context(vis)
    ck = _rms_sharded(_lin(W, ctx, f"{p}.ca.k"), W[f"{p}.ca.nk.w"], D, c.eps, allreduce).view(-1, Hl, HD)
    cv = _lin(W, ctx, f"{p}.ca.v").view(-1, Hl, HD)
    y = layer_norm(xs, W[f"{p}.n3.w"], W[f"{p}.n3.b"], c.eps)
    q = _rms_sharded(_lin(W, y, f"{p}.ca.q"), W[f"{p}.ca.nq.w"], D, c.eps, allreduce).view(-1, Hl, HD)
    a = attention(q, ck, cv).reshape(-1, Hl * HD)
    xs = xs + allreduce(_lin(W, a, f"{p}.ca.o", bias=False)) + W[f"{p}.ca.o.b"]
    # FFN over this rank's hidden columns
    y = modulate(xs, ee[3], ee[4])
    h = gelu_tanh(_lin(W, y, f"{p}.ffn.0"))
    f = allreduce(_lin(W, h, f"{p}.ffn.2", bias=False)) + W[f"{p}.ffn.2.b"]
    return xs + f * ee[5]
