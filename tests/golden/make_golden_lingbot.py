"""Generate the golden fixture that pins the LingBot oracle to the reference's own runtime code.

Run once, where a checkout of the reference (StevenCYLu/fastworld) is available:

    python tests/golden/make_golden_lingbot.py --reference <path to the fastworld checkout>

What it runs: the reference's ``StaticLingbot.__init__``, ``_consts``, ``set_prompt``,
``set_session``, ``reset``, ``_prep``, ``_cam_emb``, ``_cam_block``, ``_hoist_cam``, ``_net``,
``_rope``, ``_roll``, ``_chunk``, ``gen_chunk(graph=False)``, ``state`` and ``load``
(``fastworld/models/lingbot_v2/static.py``), unmodified, on the CPU, for 7 chunks (every KV plan
of an 18-frame window with a 6-frame sink).  The third-party pieces it calls (the LingBot/Wan
modules, the scheduler, ``flash_attn`` and the official-loop module ``engine.py``, which imports
the absent ``wan`` package) get stand-ins: ``torch.nn`` modules under the names the reference
reads, with the layer definitions of ``fastworld_b200.lingbot.param_specs`` and its seeded
weights; a scheduler holding ``lingbot.scheduler_tables``; plain softmax attention.  After
``__init__`` every bf16 buffer is switched to fp32 and the prompt is set again, so the whole
reference data flow runs in fp32.

Output ``tests/golden/lingbot_ref.pt``: per chunk the x0 latent and the plan; the window's live
prefix after the 7 chunks (sampled); a branch check (state after chunk 4, chunk 5, restore,
chunk 5 again).
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

from fastworld_b200.lingbot import LINGBOT_SMALL, scheduler_tables, synthetic_inputs, synthetic_state_dict  # noqa: E402

CFG = LINGBOT_SMALL.replace(text_len=512)     # the reference sizes its prompt K/V for 512 tokens
SEED, INPUT_SEED, N_CHUNKS = 5, 6, 7


class RMSNorm(nn.Module):
    def __init__(self, n, eps=1e-6):
        super().__init__()
        self.weight, self.eps = nn.Parameter(torch.ones(n)), eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).type_as(x) * self.weight


class Attn(nn.Module):
    def __init__(self, dim, heads):
        super().__init__()
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = RMSNorm(dim), RMSNorm(dim)
        self.num_heads, self.head_dim = heads, dim // heads


class Block(nn.Module):
    def __init__(self, c):
        super().__init__()
        D = c.dim
        self.modulation = nn.Parameter(torch.zeros(1, 6, D))
        self.self_attn, self.cross_attn = Attn(D, c.heads), Attn(D, c.heads)
        self.norm1 = nn.LayerNorm(D, eps=c.eps, elementwise_affine=False)
        self.norm2 = nn.LayerNorm(D, eps=c.eps, elementwise_affine=False)
        self.norm3 = nn.LayerNorm(D, eps=c.eps, elementwise_affine=True)
        self.ffn = nn.Sequential(nn.Linear(D, c.ffn), nn.GELU(approximate="tanh"), nn.Linear(c.ffn, D))
        self.cam_injector_layer1, self.cam_injector_layer2 = nn.Linear(D, D), nn.Linear(D, D)
        self.cam_scale_layer, self.cam_shift_layer = nn.Linear(D, D), nn.Linear(D, D)


class Head(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.modulation = nn.Parameter(torch.zeros(1, 2, c.dim))
        self.norm = nn.LayerNorm(c.dim, eps=c.eps, elementwise_affine=False)
        self.head = nn.Linear(c.dim, c.lat_ch * 4)

    def forward(self, x, e):                        # x [1, L, D], e [1, L, D]
        e = (self.modulation.unsqueeze(0) + e.unsqueeze(2)).chunk(2, dim=2)
        return self.head(self.norm(x) * (1 + e[1].squeeze(2)) + e[0].squeeze(2))


class Net(nn.Module):
    def __init__(self, c, freqs):
        super().__init__()
        D = c.dim
        self.dim, self.freq_dim, self.text_len, self.out_dim, self.patch_size = D, c.freq_dim, c.text_len, c.lat_ch, (1, 2, 2)
        self.freqs = freqs
        self.patch_embedding = nn.Conv3d(c.lat_ch + c.y_ch, D, (1, 2, 2), (1, 2, 2))
        self.text_embedding = nn.Sequential(nn.Linear(c.text_dim, D), nn.GELU(approximate="tanh"), nn.Linear(D, D))
        self.time_embedding = nn.Sequential(nn.Linear(c.freq_dim, D), nn.SiLU(), nn.Linear(D, D))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(D, 6 * D))
        self.patch_embedding_wancamctrl = nn.Linear(c.cam_ch * 4, D)
        self.c2ws_hidden_states_layer1, self.c2ws_hidden_states_layer2 = nn.Linear(D, D), nn.Linear(D, D)
        self.blocks = nn.ModuleList(Block(c) for _ in range(c.layers))
        self.head = Head(c)


def load_weights(net: Net, sd):
    got = dict(net.named_parameters())
    with torch.no_grad():
        for name, prm in got.items():
            prm.copy_(sd[name].float().view_as(prm))
    assert set(got) == set(sd), sorted(set(got) ^ set(sd))


def wan_freqs(head_dim, max_pos=1024, theta=10000.0):
    d, out = head_dim, []
    for p in (d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)):
        f = torch.outer(torch.arange(max_pos), 1.0 / torch.pow(theta, torch.arange(0, p, 2).double() / p))
        out.append(torch.polar(torch.ones_like(f), f))
    return torch.cat(out, 1)


def _attn(q, k, v):
    s = torch.einsum("blhd,bmhd->bhlm", q.float(), k.float()) / math.sqrt(q.shape[-1])
    return torch.einsum("bhlm,bmhd->blhd", torch.softmax(s, -1), v.float()).type_as(q)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.,
                           softmax_scale=None, causal=False, window_size=(-1, -1), deterministic=False):
    assert not causal and softmax_scale is None and len(cu_seqlens_q) == 2
    return _attn(q[None], k[None], v[None])[0]


def sinusoidal_embedding_1d(dim, position):
    half = dim // 2
    pos = position.type(torch.float64)
    s = torch.outer(pos, torch.pow(10000, -torch.arange(half).to(pos).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


class Scheduler:
    def __init__(self):
        sig, ts = scheduler_tables()
        self.sigmas, self.timesteps = torch.from_numpy(sig), torch.from_numpy(ts)

    def index_for_timestep(self, t, schedule_timesteps):
        idx = (schedule_timesteps == t).nonzero()
        return idx[1 if len(idx) > 1 else 0].item()

    def _sigma_to_alpha_sigma_t(self, sigma):
        return 1 - sigma, sigma


def install_fakes():
    wan = types.ModuleType("wan")
    mods = types.ModuleType("wan.modules")
    mm = types.ModuleType("wan.modules.model")
    mm.sinusoidal_embedding_1d = sinusoidal_embedding_1d
    fa = types.ModuleType("flash_attn")
    fa.flash_attn_varlen_func = flash_attn_varlen_func
    # the package __init__ imports these names from the official-loop module (engine.py:24 for the
    # window constants; the others are paths and loaders this run does not use)
    eng = types.ModuleType("fastworld.models.lingbot_v2.engine")
    eng.LOCAL_ATTN, eng.SINK = 18, 6
    for name in ("ASSETS", "CHUNK", "CKPT", "REPO", "SEED", "TIMESTEPS_INDEX", "EagerSession", "Inputs", "ex_paths",
                 "ex_prompt", "load_pipe", "official_latents", "prepare_inputs"):
        setattr(eng, name, None)
    sys.modules.update({"wan": wan, "wan.modules": mods, "wan.modules.model": mm, "flash_attn": fa,
                        "fastworld.models.lingbot_v2.engine": eng})


def sample(t: torch.Tensor, n=4096, seed=0):
    flat = t.detach().reshape(-1).double()
    g = torch.Generator().manual_seed(seed + flat.numel())
    idx = torch.randint(0, flat.numel(), (min(n, flat.numel()),), generator=g)
    return {"idx": idx, "val": flat[idx].float(), "sum": float(flat.sum()), "sumsq": float((flat * flat).sum()),
            "shape": tuple(t.shape)}


def to_f32(S):
    for nm in ("K", "V", "xk", "xv", "cam1", "camb"):
        setattr(S, nm, [t.float() for t in getattr(S, nm)])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the fastworld checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "lingbot_ref.pt"))
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    install_fakes()
    torch.set_grad_enabled(False)
    from fastworld.models.lingbot_v2 import static as ref

    c = CFG
    sd = synthetic_state_dict(c, SEED)
    net = Net(c, wan_freqs(c.head_dim))
    load_weights(net, sd)
    sch = Scheduler()
    inp = synthetic_inputs(c, N_CHUNKS, seed=INPUT_SEED, text_tokens=20)
    I = types.SimpleNamespace(
        prompt="p0", context=[inp.context.float()], noise=inp.noise.float(), y=inp.y.float(),
        plucker=inp.plucker.float(), timesteps=sch.timesteps[list(c.steps_index)],
        g_state=torch.Generator().manual_seed(inp.seed).get_state(), chunk_size=c.chunk, lat_h=c.lat_h,
        lat_w=c.lat_w, frame_seqlen=c.frame_tokens)
    pipe = types.SimpleNamespace(model=net, device=torch.device("cpu"), param_dtype=torch.bfloat16, scheduler=sch)
    S = ref.StaticLingbot(pipe, I, hoist=True, max_chunks=16)
    to_f32(S)
    S.set_prompt(I.context)
    S.reset()
    res = {"config": c.name, "text_len": c.text_len, "seed": SEED, "input_seed": INPUT_SEED, "text_tokens": 20,
           "chunks": []}
    for k in range(N_CHUNKS):
        out = S.gen_chunk(k, graph=False)
        res["chunks"].append({"k": k, "plan": S.plans[k], "x0": out.clone(), "live": S.live})
        if k == 4:
            st = S.state()
    res["window"] = {"K": [sample(t[0, :S.live * c.frame_tokens]) for t in S.K],
                     "V": [sample(t[0, :S.live * c.frame_tokens]) for t in S.V]}
    # branch: the state after chunk 4, chunk 5, then restore and chunk 5 again
    S.load(st)
    res["branch_x0"] = S.gen_chunk(5, graph=False).clone()
    torch.save(res, args.out)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
