"""Seeded synthetic weights for the MG2-shaped DiT (BASELINE: random-init weights from the seed).

The reference loads the official checkpoint into the official module tree
(``fastworld/models/mg2/model.py:39-46``); with no checkpoint available, every parameter is
drawn here from a per-tensor generator so that any subset can be regenerated on its own.
Linear and conv weights are Xavier-uniform, biases follow ``nn.Linear``'s default
U(-1/sqrt(fan_in), 1/sqrt(fan_in)), norm weights are 1 + U(-0.1, 0.1), norm biases
U(-0.1, 0.1) and adaLN modulation tables N(0, 1)/sqrt(dim) (Wan2.1 init).  All values are
rounded to bf16, the checkpoint dtype, so a CPU fp32 computation with the same tensors sees
exactly the numbers the device kernels see.

Flat names (all 2-D weights are ``[out_features, in_features]``, row-major):

====================  ===========================================  ===========================
name                  shape                                        module (Wan2.1 / MG2)
====================  ===========================================  ===========================
patch.w / patch.b     [dim, 36*1*2*2] / [dim]                      ``patch_embedding`` Conv3d
time.0.w/b time.2.w/b [dim, 256] [dim, dim]                        ``time_embedding``
tproj.w / tproj.b     [6*dim, dim]                                 ``time_projection``
img.ln0.* img.fc1.*   LN(ctx_dim), Linear(ctx_dim, ctx_dim)        ``img_emb`` (MLPProj)
img.fc2.* img.ln1.*   Linear(ctx_dim, dim), LN(dim)
head.mod head.w/b     [2, dim], [out_dim, dim]                     ``head``
b{i}.mod              [6, dim]                                     ``blocks[i].modulation``
b{i}.sa.{q,k,v,o}.*   [dim, dim]                                   ``self_attn``
b{i}.sa.nq.w/.nk.w    [dim]                                        ``norm_q`` / ``norm_k``
b{i}.n3.w / .b        [dim]                                        ``norm3``
b{i}.ca.{q,k,v,o}.*   [dim, dim]                                   ``cross_attn``
b{i}.ca.nq.w/.nk.w    [dim]
b{i}.ffn.0.* ffn.2.*  [ffn, dim] / [dim, ffn]                      ``ffn``
b{i}.am.*             see ``_action_specs``                        ``action_model``
====================  ===========================================  ===========================
"""
from __future__ import annotations

import hashlib
from typing import Dict, List, Tuple

import torch

from .config import DiTConfig

Spec = Tuple[str, Tuple[int, ...], str, int, int]   # name, shape, kind, fan_in, fan_out


def _lin(specs: List[Spec], name: str, out_f: int, in_f: int, bias: bool = True) -> None:
    specs.append((f"{name}.w", (out_f, in_f), "xavier", in_f, out_f))
    if bias:
        specs.append((f"{name}.b", (out_f,), "bias", in_f, out_f))


def _norm(specs: List[Spec], name: str, n: int, bias: bool) -> None:
    specs.append((f"{name}.w", (n,), "normw", n, n))
    if bias:
        specs.append((f"{name}.b", (n,), "normb", n, n))


def _action_specs(cfg: DiTConfig, p: str) -> List[Spec]:
    s: List[Spec] = []
    a = cfg.act_dim
    _lin(s, f"{p}.mlp1", cfg.mouse_hidden, cfg.dim + cfg.mouse_dim * cfg.pad_t)   # mouse_mlp[0]
    _lin(s, f"{p}.mlp2", cfg.mouse_hidden, cfg.mouse_hidden)                      # mouse_mlp[2]
    _norm(s, f"{p}.mln", cfg.mouse_hidden, True)                                  # mouse_mlp[3] LayerNorm
    _lin(s, f"{p}.tqkv", 3 * a, cfg.mouse_hidden)                                 # t_qkv
    _norm(s, f"{p}.mqn", cfg.act_head_dim, False)                                 # img_attn_q_norm
    _norm(s, f"{p}.mkn", cfg.act_head_dim, False)                                 # img_attn_k_norm
    _lin(s, f"{p}.pmouse", cfg.dim, a)                                            # proj_mouse
    _lin(s, f"{p}.kbe1", cfg.keyboard_hidden, cfg.keyboard_dim)                   # keyboard_embed[0]
    _lin(s, f"{p}.kbe2", cfg.keyboard_hidden, cfg.keyboard_hidden)                # keyboard_embed[2]
    _lin(s, f"{p}.mattq", a, cfg.dim)                                             # mouse_attn_q
    _lin(s, f"{p}.kbkv", 2 * a, cfg.keyboard_hidden * cfg.pad_t)                  # keyboard_attn_kv
    _norm(s, f"{p}.kqn", cfg.act_head_dim, False)                                 # key_attn_q_norm
    _norm(s, f"{p}.kkn", cfg.act_head_dim, False)                                 # key_attn_k_norm
    _lin(s, f"{p}.pkb", cfg.dim, a)                                               # proj_keyboard
    return s


def param_specs(cfg: DiTConfig) -> List[Spec]:
    d = cfg.dim
    s: List[Spec] = []
    s.append(("patch.w", (d, cfg.patch_k), "xavier", cfg.patch_k, d * 4))
    s.append(("patch.b", (d,), "bias", cfg.patch_k, d))
    _lin(s, "time.0", d, cfg.freq_dim)
    _lin(s, "time.2", d, d)
    _lin(s, "tproj", 6 * d, d)
    _norm(s, "img.ln0", cfg.ctx_dim, True)
    _lin(s, "img.fc1", cfg.ctx_dim, cfg.ctx_dim)
    _lin(s, "img.fc2", d, cfg.ctx_dim)
    _norm(s, "img.ln1", d, True)
    s.append(("head.mod", (2, d), "mod", d, d))
    _lin(s, "head", cfg.out_dim, d)
    for i in range(cfg.layers):
        p = f"b{i}"
        s.append((f"{p}.mod", (6, d), "mod", d, d))
        for nm in ("q", "k", "v", "o"):
            _lin(s, f"{p}.sa.{nm}", d, d)
        _norm(s, f"{p}.sa.nq", d, False)
        _norm(s, f"{p}.sa.nk", d, False)
        _norm(s, f"{p}.n3", d, True)
        for nm in ("q", "k", "v", "o"):
            _lin(s, f"{p}.ca.{nm}", d, d)
        _norm(s, f"{p}.ca.nq", d, False)
        _norm(s, f"{p}.ca.nk", d, False)
        _lin(s, f"{p}.ffn.0", cfg.ffn, d)
        _lin(s, f"{p}.ffn.2", d, cfg.ffn)
        if i in cfg.action_blocks:
            s.extend(_action_specs(cfg, f"{p}.am"))
    return s


def _tensor_seed(seed: int, name: str) -> int:
    h = hashlib.sha1(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


_COL_PARALLEL = (".sa.q.", ".sa.k.", ".sa.v.", ".ca.q.", ".ca.k.", ".ca.v.", ".sa.nq.", ".sa.nk.",
                 ".ca.nq.", ".ca.nk.")
_ROW_PARALLEL = (".sa.o.w", ".ca.o.w")


def shard_tensor(cfg: DiTConfig, name: str, t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's part of one flat-named tensor under tensor parallelism over `world` ranks.

    Attention is split by heads: the q/k/v (self and cross) rows and q/k RMSNorm weights of
    heads [rank * heads / world, ...) and the matching input columns of the output
    projections.  The FFN is split by hidden columns: rows of ffn.0, input columns of ffn.2.
    Output-projection biases, norms outside attention, embeddings, the head and the adaLN
    tables stay whole (replicated)."""
    if world == 1 or not name.startswith("b"):
        return t
    dl, fl = cfg.dim // world, cfg.ffn // world
    if any(k in name for k in _COL_PARALLEL):
        return t[rank * dl:(rank + 1) * dl]
    if name.endswith(_ROW_PARALLEL):
        return t[:, rank * dl:(rank + 1) * dl]
    if ".ffn.0." in name:
        return t[rank * fl:(rank + 1) * fl]
    if name.endswith(".ffn.2.w"):
        return t[:, rank * fl:(rank + 1) * fl]
    return t


def shard_state_dict(cfg: DiTConfig, sd: Dict[str, torch.Tensor], rank: int, world: int) -> Dict[str, torch.Tensor]:
    """:func:`shard_tensor` over a whole state dict (contiguous copies of the local parts)."""
    if cfg.heads % world or cfg.ffn % world:
        raise ValueError(f"{world} ranks do not divide {cfg.heads} heads / ffn {cfg.ffn}")
    return {k: shard_tensor(cfg, k, v, rank, world).contiguous() for k, v in sd.items()}


def synthetic_state_dict(cfg: DiTConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                         shard=None) -> Dict[str, torch.Tensor]:
    """Seeded weights, one generator per tensor. Values depend on the device's RNG.

    ``shard=(rank, world)`` keeps only this rank's tensor-parallel part of each tensor as it is
    drawn (same values as sharding the full dict; the full model is never resident)."""
    cfg.validate()
    out: Dict[str, torch.Tensor] = {}
    for name, shape, kind, fi, fo in param_specs(cfg):
        g = torch.Generator(device=device).manual_seed(_tensor_seed(seed, name))
        if kind == "xavier":
            bound = (6.0 / (fi + fo)) ** 0.5
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) * bound
        elif kind == "bias":
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) / fi ** 0.5
        elif kind == "normw":
            t = 1 + (torch.rand(shape, generator=g, device=device) * 2 - 1) * 0.1
        elif kind == "normb":
            t = (torch.rand(shape, generator=g, device=device) * 2 - 1) * 0.1
        elif kind == "mod":
            t = torch.randn(shape, generator=g, device=device) / cfg.dim ** 0.5
        else:  # pragma: no cover
            raise ValueError(kind)
        t = t.to(dtype)
        if shard is not None:
            t = shard_tensor(cfg, name, t, *shard).contiguous()
        out[name] = t
    return out


def state_dict_bytes(cfg: DiTConfig) -> int:
    n = 0
    for _, shape, *_ in param_specs(cfg):
        k = 1
        for x in shape:
            k *= x
        n += k
    return 2 * n
