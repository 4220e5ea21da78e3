"""Generate the golden fixtures that pin the CPU oracle to the reference's own code.

Run once, where a checkout of the reference (StevenCYLu/fastworld) is available:

    python tests/golden/make_golden.py --reference <path to the fastworld checkout>

What it runs: the reference's ``StaticMG.__init__``, ``_prep``, ``_net``, ``_action``,
``_cross``, ``_rope``, ``_chunk``, ``gen_chunk(graph=False)``, ``prefill(graph=False)``,
``state`` and ``load`` (``fastworld/models/mg2/static.py``), unmodified, on the CPU.  The
third-party pieces it calls (the Matrix-Game-2 ``wan`` modules, ``flash_attn`` and the
scheduler wrapper) are absent from the reference, so this script supplies stand-ins written
as ``torch.nn`` modules that implement the layer definitions pinned in
``fastworld_b200/config.py`` (plain softmax attention in place of flash-attn).  After
``__init__`` every bf16 buffer is switched to fp32, so the whole reference data flow runs
in fp32 and the oracle can be compared at fp32 precision.

Outputs (``tests/golden/tiny_ref.pt``): per chunk of a 3-chunk path (chunk 0 is the
"first" graph, chunks 1-2 steady) the prepared inputs (``gm``, ``kc``, a sample of ``fi``)
and a sample of the output latent; the session state after the rollout; a branch check
(save, alternative chunk, restore, continue) and one prefill.  Samples are fixed index sets
plus float64 sum and sum of squares of the full tensor.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
import types

import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from fastworld_b200.config import TINY  # noqa: E402
from fastworld_b200.prep import CAM, synthetic_image  # noqa: E402
from fastworld_b200.weights import synthetic_state_dict  # noqa: E402

SEED, IMG_SEED, N_SAMPLE = 1, 7, 4096


# --------------------------------------------------------------------- stand-in modules
class RMSNorm(nn.Module):
    def __init__(self, n, eps=1e-6):
        super().__init__()
        self.weight, self.eps = nn.Parameter(torch.ones(n)), eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).type_as(x) * self.weight


class LN(nn.LayerNorm):
    def __init__(self, n, affine, eps):
        super().__init__(n, eps=eps, elementwise_affine=affine)


class Attn(nn.Module):
    def __init__(self, dim, heads):
        super().__init__()
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = RMSNorm(dim), RMSNorm(dim)
        self.num_heads, self.head_dim = heads, dim // heads


class Action(nn.Module):
    def __init__(self, c, cos, sin):
        super().__init__()
        a = c.act_dim
        self.heads_num, self.vae_time_compression_ratio, self.windows_size = c.act_heads, c.time_ratio, c.window
        self.freqs_cos, self.freqs_sin = cos, sin
        self.mouse_mlp = nn.Sequential(nn.Linear(c.dim + c.mouse_dim * c.pad_t, c.mouse_hidden),
                                       nn.GELU(approximate="tanh"), nn.Linear(c.mouse_hidden, c.mouse_hidden),
                                       nn.LayerNorm(c.mouse_hidden))
        self.t_qkv = nn.Linear(c.mouse_hidden, 3 * a)
        self.img_attn_q_norm, self.img_attn_k_norm = RMSNorm(c.act_head_dim), RMSNorm(c.act_head_dim)
        self.proj_mouse = nn.Linear(a, c.dim)
        self.keyboard_embed = nn.Sequential(nn.Linear(c.keyboard_dim, c.keyboard_hidden), nn.SiLU(),
                                            nn.Linear(c.keyboard_hidden, c.keyboard_hidden))
        self.mouse_attn_q = nn.Linear(c.dim, a)
        self.keyboard_attn_kv = nn.Linear(c.keyboard_hidden * c.pad_t, 2 * a)
        self.key_attn_q_norm, self.key_attn_k_norm = RMSNorm(c.act_head_dim), RMSNorm(c.act_head_dim)
        self.proj_keyboard = nn.Linear(a, c.dim)


class Block(nn.Module):
    def __init__(self, c, has_action, cos, sin):
        super().__init__()
        self.modulation = nn.Parameter(torch.zeros(1, 6, c.dim))
        self.self_attn, self.cross_attn = Attn(c.dim, c.heads), Attn(c.dim, c.heads)
        self.norm1, self.norm2 = LN(c.dim, False, c.eps), LN(c.dim, False, c.eps)
        self.norm3 = LN(c.dim, True, c.eps)
        self.ffn = nn.Sequential(nn.Linear(c.dim, c.ffn), nn.GELU(approximate="tanh"), nn.Linear(c.ffn, c.dim))
        self.action_model = Action(c, cos, sin) if has_action else None


class Head(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.modulation = nn.Parameter(torch.zeros(1, 2, c.dim))
        self.norm = LN(c.dim, False, c.eps)
        self.head = nn.Linear(c.dim, c.out_dim)
        self.F, self.S = c.frames, c.tok_per_frame

    def forward(self, x, e):                      # x [1, L, dim], e [1, F, 1, dim]
        sh, sc = (self.modulation.unsqueeze(1) + e).chunk(2, dim=2)
        y = self.norm(x).unflatten(1, (self.F, self.S)) * (1 + sc) + sh
        return self.head(y.flatten(1, 2))


class Net(nn.Module):
    def __init__(self, c, freqs, cos, sin):
        super().__init__()
        self.c, self.dim, self.freq_dim, self.freqs = c, c.dim, c.freq_dim, freqs
        self.patch_embedding = nn.Conv3d(c.lat_ch + c.cond_ch, c.dim, c.patch, c.patch)
        self.time_embedding = nn.Sequential(nn.Linear(c.freq_dim, c.dim), nn.SiLU(), nn.Linear(c.dim, c.dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(c.dim, 6 * c.dim))
        self.img_emb = nn.Sequential(nn.LayerNorm(c.ctx_dim), nn.Linear(c.ctx_dim, c.ctx_dim), nn.GELU(),
                                     nn.Linear(c.ctx_dim, c.dim), nn.LayerNorm(c.dim))
        self.blocks = nn.ModuleList(Block(c, i in c.action_blocks, cos, sin) for i in range(c.layers))
        self.head = Head(c)

    def unpatchify(self, out, grid):
        f, h, w = (int(v) for v in grid)
        c = self.c
        u = out[0][: f * h * w].view(f, h, w, *c.patch, c.lat_ch)
        u = torch.einsum("fhwpqrc->cfphqwr", u).reshape(c.lat_ch, f * c.patch[0], h * c.patch[1], w * c.patch[2])
        return u[None]


def load_weights(net: Net, sd, c):
    W = {k: v.float() for k, v in sd.items()}
    P = {}

    def lin(mod, name):
        P[id(mod.weight)] = W[f"{name}.w"].view_as(mod.weight)
        P[id(mod.bias)] = W[f"{name}.b"]

    def norm(mod, name):
        P[id(mod.weight)] = W[f"{name}.w"]
        if getattr(mod, "bias", None) is not None:
            P[id(mod.bias)] = W[f"{name}.b"]

    lin(net.patch_embedding, "patch")
    lin(net.time_embedding[0], "time.0"); lin(net.time_embedding[2], "time.2")
    lin(net.time_projection[1], "tproj")
    norm(net.img_emb[0], "img.ln0"); lin(net.img_emb[1], "img.fc1"); lin(net.img_emb[3], "img.fc2")
    norm(net.img_emb[4], "img.ln1")
    P[id(net.head.modulation)] = W["head.mod"][None]
    lin(net.head.head, "head")
    for i, b in enumerate(net.blocks):
        p = f"b{i}"
        P[id(b.modulation)] = W[f"{p}.mod"][None]
        for an, mod in (("sa", b.self_attn), ("ca", b.cross_attn)):
            for nm in "qkvo":
                lin(getattr(mod, nm), f"{p}.{an}.{nm}")
            norm(mod.norm_q, f"{p}.{an}.nq"); norm(mod.norm_k, f"{p}.{an}.nk")
        norm(b.norm3, f"{p}.n3")
        lin(b.ffn[0], f"{p}.ffn.0"); lin(b.ffn[2], f"{p}.ffn.2")
        a = b.action_model
        if a is not None:
            q = f"{p}.am"
            lin(a.mouse_mlp[0], f"{q}.mlp1"); lin(a.mouse_mlp[2], f"{q}.mlp2"); norm(a.mouse_mlp[3], f"{q}.mln")
            lin(a.t_qkv, f"{q}.tqkv"); norm(a.img_attn_q_norm, f"{q}.mqn"); norm(a.img_attn_k_norm, f"{q}.mkn")
            lin(a.proj_mouse, f"{q}.pmouse")
            lin(a.keyboard_embed[0], f"{q}.kbe1"); lin(a.keyboard_embed[2], f"{q}.kbe2")
            lin(a.mouse_attn_q, f"{q}.mattq"); lin(a.keyboard_attn_kv, f"{q}.kbkv")
            norm(a.key_attn_q_norm, f"{q}.kqn"); norm(a.key_attn_k_norm, f"{q}.kkn")
            lin(a.proj_keyboard, f"{q}.pkb")
    n = 0
    with torch.no_grad():
        for prm in net.parameters():
            prm.copy_(P[id(prm)])
            n += 1
    assert n == len(P), (n, len(P))


# --------------------------------------------------------------------- stand-in libraries
def _attn(q, k, v):                                   # [B, L, H, D]
    s = torch.einsum("blhd,bmhd->bhlm", q.float(), k.float()) / math.sqrt(q.shape[-1])
    return torch.einsum("bhlm,bmhd->blhd", torch.softmax(s, -1), v.float()).type_as(q)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.,
                           softmax_scale=None, causal=False, window_size=(-1, -1), deterministic=False):
    assert not causal and softmax_scale is None and len(cu_seqlens_q) == 2
    return _attn(q[None], k[None], v[None])[0]


def flash_attn_func(q, k, v):
    return _attn(q, k, v)


def sinusoidal_embedding_1d(dim, position):
    half = dim // 2
    pos = position.type(torch.float64)
    s = torch.outer(pos, torch.pow(10000, -torch.arange(half).to(pos).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


def rotate_half(x):
    xr = x.float().reshape(*x.shape[:-1], -1, 2)
    return torch.stack([-xr[..., 1], xr[..., 0]], dim=-1).flatten(-2)


class Scheduler:
    sigmas = torch.linspace(1, 0, 1001)[:-1]
    timesteps = sigmas * 1000

    def add_noise(self, x, noise, t):
        sg = (t.double() / 1000).reshape(-1, 1, 1, 1)
        return ((1 - sg) * x.double() + sg * noise.double()).type_as(noise)


class Generator:
    def __init__(self, net, sch):
        self.model, self.scheduler = net, sch

    def _convert_flow_pred_to_x0(self, flow_pred, xt, timestep):
        sg = (timestep.double() / 1000).reshape(-1, 1, 1, 1)
        return (xt.double() - sg * flow_pred.double()).to(flow_pred.dtype)


def install_fakes():
    wan = types.ModuleType("wan")
    mods = types.ModuleType("wan.modules")
    mm = types.ModuleType("wan.modules.model")
    mm.sinusoidal_embedding_1d = sinusoidal_embedding_1d
    pe = types.ModuleType("wan.modules.posemb_layers")
    pe.rotate_half = rotate_half
    fa = types.ModuleType("flash_attn")
    fa.flash_attn_varlen_func, fa.flash_attn_func = flash_attn_varlen_func, flash_attn_func
    sys.modules.update({"wan": wan, "wan.modules": mods, "wan.modules.model": mm,
                        "wan.modules.posemb_layers": pe, "flash_attn": fa})


def wan_freqs(c):
    """Wan ``rope_params`` for (t, h, w) concatenated: complex128 [max_frames, head_dim // 2]."""
    d, out = c.head_dim, []
    for p in (d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)):
        f = torch.outer(torch.arange(c.max_frames), 1.0 / torch.pow(c.rope_theta, torch.arange(0, p, 2).double() / p))
        out.append(torch.polar(torch.ones_like(f), f))
    return torch.cat(out, 1)


def action_freqs(c):
    d = c.act_head_dim
    f = torch.outer(torch.arange(c.max_frames).double(), 1.0 / torch.pow(c.rope_theta, torch.arange(0, d, 2).double() / d))
    return f.cos().float().repeat_interleave(2, 1), f.sin().float().repeat_interleave(2, 1)


# --------------------------------------------------------------------- helpers
def sample(t: torch.Tensor, n=N_SAMPLE, seed=0):
    flat = t.detach().reshape(-1).double()
    g = torch.Generator().manual_seed(seed + flat.numel())
    idx = torch.randint(0, flat.numel(), (min(n, flat.numel()),), generator=g)
    return {"idx": idx, "val": flat[idx].float(), "sum": float(flat.sum()), "sumsq": float((flat * flat).sum()),
            "shape": tuple(t.shape)}


def to_f32(S):
    S.hk = [t.float() for t in S.hk]; S.hv = [t.float() for t in S.hv]
    for nm in ("mk", "mv", "kk", "kv"):
        setattr(S, nm, {i: t.float() for i, t in getattr(S, nm).items()})
    for nm in ("x_in", "cc", "vis", "gm", "kc", "out", "lat_in"):
        setattr(S, nm, getattr(S, nm).float())
    S.noise = [t.float() for t in S.noise]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the fastworld checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "tiny_ref.pt"))
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    install_fakes()
    torch.set_grad_enabled(False)
    from fastworld.models.mg2 import static as ref_static
    from fastworld.models.mg2.model import path_seed as ref_path_seed

    c = TINY
    sd = synthetic_state_dict(c, SEED)
    cos, sin = action_freqs(c)
    net = Net(c, wan_freqs(c), cos, sin)
    load_weights(net, sd, c)
    sch = Scheduler()
    M = types.SimpleNamespace(dev="cpu", steps=list(c.steps), images={"img0": synthetic_image(c, IMG_SEED, 8)})
    M.p = types.SimpleNamespace(generator=Generator(net, sch), scheduler=sch)
    assert ref_static.FPB == c.frames and ref_static.TOK == c.tok_per_frame
    S = ref_static.StaticMG(M)
    to_f32(S)

    path = [("img0", ("w", "u")), ("img0", ("a", "l")), ("img0", ("q", "i")), ("img0", ("d", "j"))]
    res = {"config": c.name, "seed": SEED, "img_seed": IMG_SEED, "path": path, "chunks": []}
    for k in range(3):
        out = S.gen_chunk(path, k, graph=False)
        res["chunks"].append({"k": k, "path_seed": ref_path_seed(path[:k + 1]), "gm": S.gm[0].clone(),
                              "kc": S.kc[0].clone(), "fi": sample(torch.view_as_real(S.fi)),
                              "x_in": sample(S.x_in), "noise": [sample(t) for t in S.noise],
                              "out": sample(out)})
    res["state"] = {"hk": [sample(t) for t in S.hk], "hv": [sample(t) for t in S.hv],
                    "mk": {i: sample(t) for i, t in S.mk.items()}, "mv": {i: sample(t) for i, t in S.mv.items()},
                    "kk": {i: sample(t) for i, t in S.kk.items()}, "kv": {i: sample(t) for i, t in S.kv.items()}}
    # branch: save after chunk 2, run an alternative chunk 3, restore, run the original chunk 3
    st = S.state()
    alt = path[:3] + [("img0", ("s", "k"))]
    S.gen_chunk(alt, 3, graph=False)
    S.load(st)
    res["branch_out"] = sample(S.gen_chunk(path, 3, graph=False))
    # prefill: advance over a known latent (chunk 3 of the path) from the restored state
    S.load(st)
    lat = S.out.clone()
    S.prefill(lat, path, 3, graph=False)
    res["prefill_lat"] = sample(lat)
    res["prefill_hk0"] = sample(S.hk[0])
    res["cam_i"] = CAM["i"]
    torch.save(res, args.out)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
