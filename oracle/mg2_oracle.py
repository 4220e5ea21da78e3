"""CPU oracle for the Matrix-Game-2-shaped chunk forward.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it.  The product path (``fastworld_b200``)
runs hand-written sm_100a kernels and fails loudly when its CUDA library is missing.

It restates, op for op, the reference runtime's forward in PyTorch fp32 on the CPU:

* ``StaticMG._net``    fastworld/models/mg2/static.py:194-230   -> :meth:`Oracle.net`
* ``StaticMG._chunk``  static.py:232-242                        -> :meth:`Oracle.chunk`
* ``StaticMG._prefill`` static.py:244-245                       -> :meth:`Oracle.prefill`
* ``StaticMG._rope``   static.py:130-133 (fp64 complex)          -> :func:`apply_rope`
* ``StaticMG._arot``   static.py:135-136                        -> :func:`apply_action_rope`
* ``StaticMG._action`` static.py:145-185                        -> :meth:`Oracle.action`
* ``StaticMG._cross``  static.py:187-192                        -> :meth:`Oracle.cross`
* RoPE table ``fi``    static.py:113-118                        -> :func:`rope_table`

The module semantics of the (un-vendored) official Wan/Matrix-Game-2 layers are the ones
pinned in ``fastworld_b200.config``.  Interface tensors that the reference keeps in bf16
(latents between denoising steps, history K/V, action state) are rounded to bf16 here too;
everything else is fp32 unless ``emulate_bf16=True``, which also rounds every tensor the
reference holds in bf16 (Linear outputs, attention inputs/outputs, norm outputs).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own ``StaticMG._prep``,
``_net`` and ``_chunk`` (imported from the reference checkout) on the CPU with fp32 buffers
and stand-in modules of the same definitions, and stores sampled outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against them.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence

import torch

F32 = torch.float32
EPS_LN_DEFAULT = 1e-5       # nn.LayerNorm default (img_emb, mouse_mlp)


def bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(x.dtype)


# ----------------------------------------------------------------------------- tables
def rope_freqs(head_dim: int, max_pos: int = 1024, theta: float = 10000.0) -> torch.Tensor:
    """``net.freqs``: Wan rope_params for (t, h, w), complex128 [max_pos, head_dim // 2]."""
    d = head_dim
    parts = [d - 4 * (d // 6), 2 * (d // 6), 2 * (d // 6)]
    out = []
    for p in parts:
        inv = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64),
                              torch.arange(0, p, 2, dtype=torch.float64) / p)
        ang = torch.outer(torch.arange(max_pos, dtype=torch.float64), inv)
        out.append(torch.polar(torch.ones_like(ang), ang))
    return torch.cat(out, dim=1)


def rope_table(cfg, k: int, freqs: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-token RoPE multipliers of chunk k, complex128 [L, head_dim // 2] (static.py:113-118)."""
    if freqs is None:
        freqs = rope_freqs(cfg.head_dim, cfg.max_frames, cfg.rope_theta)
    ft, fh, fw = freqs.split(list(cfg.rope_split), dim=1)
    f, h, w, s = cfg.frames, cfg.th, cfg.tw, cfg.frames * k
    tab = torch.cat([ft[s:s + f].view(f, 1, 1, -1).expand(f, h, w, -1),
                     fh[:h].view(1, h, 1, -1).expand(f, h, w, -1),
                     fw[:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1)
    return tab.reshape(f * h * w, -1)


def apply_rope(x: torch.Tensor, fi: torch.Tensor) -> torch.Tensor:
    """x [L, H, D] -> complex rotation of (x[2i], x[2i+1]) pairs in fp64 (static.py:130-133)."""
    L, H, D = x.shape
    xc = torch.view_as_complex(x.to(torch.float64).reshape(L, H, D // 2, 2))
    return torch.view_as_real(xc * fi[:, None, :]).reshape(L, H, D).to(x.dtype)


def action_rope_tables(cfg) -> (torch.Tensor, torch.Tensor):
    """``freqs_cos/freqs_sin`` of the action module: fp32 [max_frames, act_head_dim], each
    frequency repeated for the (even, odd) pair it rotates."""
    d = cfg.act_head_dim
    inv = 1.0 / torch.pow(torch.tensor(cfg.rope_theta, dtype=torch.float64),
                          torch.arange(0, d, 2, dtype=torch.float64) / d)
    ang = torch.outer(torch.arange(cfg.max_frames, dtype=torch.float64), inv)
    return (ang.cos().repeat_interleave(2, dim=1).float(), ang.sin().repeat_interleave(2, dim=1).float())


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """(x0, x1) pairs -> (-x1, x0)."""
    xr = x.reshape(*x.shape[:-1], -1, 2)
    return torch.stack([-xr[..., 1], xr[..., 0]], dim=-1).reshape(x.shape)


def apply_action_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``_arot`` (static.py:135-136): x * cos + rotate_half(x) * sin, fp32."""
    xf = x.float()
    return (xf * cos + rotate_half(xf) * sin).to(x.dtype)


def sinusoid(freq_dim: int, t: float) -> torch.Tensor:
    """Wan ``sinusoidal_embedding_1d`` of one timestep, fp64 -> fp32 [freq_dim]."""
    half = freq_dim // 2
    pos = torch.tensor([float(t)], dtype=torch.float64)
    s = torch.outer(pos, torch.pow(torch.tensor(10000.0, dtype=torch.float64),
                                   -torch.arange(half, dtype=torch.float64).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)[0].float()


def sigma_of(t: float) -> float:
    """Flow-matching sigma of a (possibly warped, float) timestep: t / 1000."""
    return float(t) / 1000.0


# ----------------------------------------------------------------------------- primitives
def layer_norm(x, w=None, b=None, eps=1e-6):
    return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), w, b, eps)


def rms_norm(x, w, eps=1e-6):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w


def gelu_tanh(x):
    return torch.nn.functional.gelu(x, approximate="tanh")


def gelu_erf(x):
    return torch.nn.functional.gelu(x)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Non-causal softmax attention. q [..., Lq, H, D], k/v [..., Lk, H, D] -> [..., Lq, H, D]."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    qh, kh, vh = (t.transpose(-3, -2).float() for t in (q, k, v))   # [..., H, L, D]
    out = torch.empty_like(qh)
    step = 2
    for h0 in range(0, qh.shape[-3], step):
        sl = (Ellipsis, slice(h0, h0 + step), slice(None), slice(None))
        s = torch.matmul(qh[sl], kh[sl].transpose(-1, -2)) * scale
        out[sl] = torch.matmul(torch.softmax(s, dim=-1), vh[sl])
    return out.transpose(-3, -2)


# ----------------------------------------------------------------------------- oracle
class Oracle:
    """fp32 CPU restatement of the chunk forward for one session."""

    def __init__(self, cfg, sd: Dict[str, torch.Tensor], emulate_bf16: bool = False,
                 round_interface: bool = True):
        cfg.validate()
        self.cfg = cfg
        self.W = {k: v.detach().to("cpu", F32) for k, v in sd.items()}
        self.emu = emulate_bf16
        self.ri = round_interface
        self.freqs = rope_freqs(cfg.head_dim, cfg.max_frames, cfg.rope_theta)
        self.acos_full, self.asin_full = action_rope_tables(cfg)

    # -- helpers
    def r(self, x):
        return bf16(x) if self.emu else x

    def i(self, x):
        """Rounding of an interface tensor (latent, history K/V, action state)."""
        return bf16(x) if self.ri else x

    def lin(self, x, name, bias=True):
        y = torch.matmul(x, self.W[f"{name}.w"].t())
        if bias and f"{name}.b" in self.W:
            y = y + self.W[f"{name}.b"]
        return self.r(y)

    # -- state
    def new_state(self) -> Dict[str, object]:
        c = self.cfg
        L, H, D = c.tokens, c.heads, c.head_dim
        W = c.hist_chunks   # history window: W slots of one chunk's keys
        st = {"hk": torch.zeros(c.layers, W * L, H, D), "hv": torch.zeros(c.layers, W * L, H, D),
              "mk": {}, "mv": {}, "kk": {}, "kv": {}}
        for i in c.action_blocks:
            st["mk"][i] = torch.zeros(c.tok_per_frame, c.frames, c.act_heads, c.act_head_dim)
            st["mv"][i] = torch.zeros_like(st["mk"][i])
            st["kk"][i] = torch.zeros(1, c.frames, c.act_heads, c.act_head_dim)
            st["kv"][i] = torch.zeros_like(st["kk"][i])
        return st

    # -- embeddings
    def time_embed(self, t: float):
        """e [dim] and e0 [6, dim] of one timestep (static.py:199-200; the forward uses int(t))."""
        s = sinusoid(self.cfg.freq_dim, int(t))
        h = torch.nn.functional.silu(self.lin(s, "time.0"))
        e = self.lin(h, "time.2")
        e0 = self.lin(torch.nn.functional.silu(e), "tproj").view(6, self.cfg.dim)
        return e, e0

    def context(self, vis: torch.Tensor) -> torch.Tensor:
        """``img_emb(vis)`` (static.py:201): LN -> Linear -> GELU -> Linear -> LN."""
        W = self.W
        x = self.r(layer_norm(vis.float(), W["img.ln0.w"], W["img.ln0.b"], EPS_LN_DEFAULT))
        x = self.r(gelu_erf(self.lin(x, "img.fc1")))
        x = self.lin(x, "img.fc2")
        return self.r(layer_norm(x, W["img.ln1.w"], W["img.ln1.b"], EPS_LN_DEFAULT))

    def patch_embed(self, x: torch.Tensor, cc: torch.Tensor) -> torch.Tensor:
        """Conv3d(36 -> dim, k = s = (1, 2, 2)) on cat([x, cc]) (static.py:197-198) -> [L, dim]."""
        c = self.cfg
        xin = torch.cat([x.float(), cc.float()], 0)                          # [36, F, H, W]
        C = xin.shape[0]
        t = xin.reshape(C, c.frames, c.th, 2, c.tw, 2).permute(1, 2, 4, 0, 3, 5)
        return self.lin(t.reshape(c.tokens, C * 4), "patch")

    def unpatchify(self, out: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        u = out.view(c.frames, c.th, c.tw, 1, 2, 2, c.lat_ch)
        return u.permute(6, 0, 3, 1, 4, 2, 5).reshape(c.lat_ch, c.frames, c.lat_h, c.lat_w)

    # -- blocks
    def cross(self, i: int, x: torch.Tensor, ctx_kv) -> torch.Tensor:
        """``_cross`` (static.py:187-192)."""
        c, p = self.cfg, f"b{i}.ca"
        q = self.r(rms_norm(self.lin(x, f"{p}.q"), self.W[f"{p}.nq.w"], c.eps)).view(-1, c.heads, c.head_dim)
        k, v = ctx_kv
        return self.lin(self.r(attention(q, k, v)).reshape(-1, c.dim), f"{p}.o")

    def cross_kv(self, i: int, context: torch.Tensor):
        c, p = self.cfg, f"b{i}.ca"
        k = self.r(rms_norm(self.lin(context, f"{p}.k"), self.W[f"{p}.nk.w"], c.eps))
        v = self.lin(context, f"{p}.v")
        return k.view(-1, c.heads, c.head_dim), v.view(-1, c.heads, c.head_dim)

    def keyboard_kv(self, i: int, kc: torch.Tensor, s: int):
        """Keyboard K/V of one block (static.py:165-172): embed -> windows -> kv -> norm -> RoPE."""
        c, p, W = self.cfg, f"b{i}.am", self.W
        ke = self.lin(torch.nn.functional.silu(self.lin(kc.float(), f"{p}.kbe1")), f"{p}.kbe2")   # [kc_len, Kh]
        r, pt = c.time_ratio, c.pad_t
        gk = torch.stack([ke[r * (f - c.window) + pt: f * r + pt] for f in range(c.frames)], 0)
        kv = self.lin(gk.reshape(c.frames, -1), f"{p}.kbkv").view(c.frames, 2, c.act_heads, c.act_head_dim)
        k = self.r(rms_norm(kv[:, 0], W[f"{p}.kkn.w"], c.eps))
        cos, sin = self.acos_full[s:s + c.frames, None, :], self.asin_full[s:s + c.frames, None, :]
        k = self.r(apply_action_rope(k, cos, sin))
        return k[None], kv[None, :, 1]                                       # [1, F, AH, 64]

    def action(self, i: int, xs: torch.Tensor, st, first: bool, write: bool, gm, kc, s: int):
        """``_action`` (static.py:145-185); xs [L, dim] token order (f, s)."""
        c, p, W = self.cfg, f"b{i}.am", self.W
        F, S, AH, AD = c.frames, c.tok_per_frame, c.act_heads, c.act_head_dim
        h = self.r(xs).view(F, S, c.dim).transpose(0, 1)                    # [S, F, C]
        g = gm.float().reshape(F, -1)[None].expand(S, F, -1)                  # [S, F, pad_t*2]
        m = self.r(gelu_tanh(self.lin(torch.cat([h, g], -1), f"{p}.mlp1")))
        m = self.lin(m, f"{p}.mlp2")
        m = self.r(layer_norm(m, W[f"{p}.mln.w"], W[f"{p}.mln.b"], EPS_LN_DEFAULT))
        qkv = self.lin(m, f"{p}.tqkv").view(S, F, 3, AH, AD)
        q = self.r(rms_norm(qkv[:, :, 0], W[f"{p}.mqn.w"], c.eps))
        k = self.r(rms_norm(qkv[:, :, 1], W[f"{p}.mkn.w"], c.eps))
        v = qkv[:, :, 2]
        cos, sin = self.acos_full[s:s + F, None, :], self.asin_full[s:s + F, None, :]
        q, k = self.r(apply_action_rope(q, cos, sin)), self.r(apply_action_rope(k, cos, sin))
        if first:
            Km, Vm = k, v
        else:
            Km, Vm = torch.cat([st["mk"][i], k], 1), torch.cat([st["mv"][i], v], 1)
        a = self.r(attention(q, Km, Vm))                                     # [S, F, AH, AD]
        if write:
            st["mk"][i], st["mv"][i] = self.i(k), self.i(v)
        a = a.transpose(0, 1).reshape(F * S, AH * AD)
        hs = h.transpose(0, 1).reshape(F * S, c.dim) + self.lin(a, f"{p}.pmouse")
        hs = self.r(hs)
        # keyboard branch
        kk_cur, kv_cur = self.keyboard_kv(i, kc, s)
        mq = self.lin(hs, f"{p}.mattq").view(F * S, AH, AD)
        q = self.r(rms_norm(mq, W[f"{p}.kqn.w"], c.eps))
        q = q.view(F, S, AH, AD).transpose(0, 1)                              # [S, F, AH, AD]
        q = self.r(apply_action_rope(q, cos, sin))
        if first:
            Kk, Vk = kk_cur, kv_cur
        else:
            Kk, Vk = torch.cat([st["kk"][i], kk_cur], 1), torch.cat([st["kv"][i], kv_cur], 1)
        if write:
            st["kk"][i], st["kv"][i] = self.i(kk_cur), self.i(kv_cur)
        a = self.r(attention(q, Kk.expand(S, -1, -1, -1), Vk.expand(S, -1, -1, -1)))
        a = a.transpose(0, 1).reshape(F * S, AH * AD)
        return hs + self.lin(a, f"{p}.pkb")

    def block(self, i: int, xs, e0, fi, st, first: bool, write: bool, ctx_kv, gm=None, kc=None, s=0, taps=None):
        """One transformer block of ``_net`` (static.py:203-225).  ``taps`` (a dict) receives
        the intermediates the engine's block tap copies (same names)."""
        c, p, W = self.cfg, f"b{i}", self.W
        F, S = c.frames, c.tok_per_frame
        ee = (W[f"{p}.mod"][None] + e0).unbind(1)                            # 6 x [F, dim]
        tap = taps.__setitem__ if taps is not None else (lambda k, v: None)
        tap("xs_in", xs)

        def per_frame(x, fn):
            return fn(x.view(F, S, c.dim)).reshape(F * S, c.dim)

        y_in = self.r(per_frame(layer_norm(xs, eps=c.eps), lambda t: t * (1 + ee[1][:, None]) + ee[0][:, None]))
        q = self.r(rms_norm(self.lin(y_in, f"{p}.sa.q"), W[f"{p}.sa.nq.w"], c.eps)).view(-1, c.heads, c.head_dim)
        k = self.r(rms_norm(self.lin(y_in, f"{p}.sa.k"), W[f"{p}.sa.nk.w"], c.eps)).view(-1, c.heads, c.head_dim)
        v = self.lin(y_in, f"{p}.sa.v").view(-1, c.heads, c.head_dim)
        rq, rk = self.r(apply_rope(q, fi)), self.i(apply_rope(k, fi))
        v = self.i(v)
        tap("q", rq)
        tap("k", rk)
        tap("v", v)
        L, Wn, k_idx = c.tokens, c.hist_chunks, s // c.frames
        # keys: the filled history slots (one chunk for MG2, static.py:213-216), then the
        # current chunk; with a window of Wn > 1 chunks, chunk k has min(k, Wn) filled slots
        n0 = L if Wn == 1 else min(k_idx, Wn) * L
        if first:
            y = attention(rq, rk, v)
        else:
            y = attention(rq, torch.cat([st["hk"][i][:n0], rk], 0), torch.cat([st["hv"][i][:n0], v], 0))
        if write:   # ring slot k % Wn (static.py:217-218 for Wn = 1)
            sl = slice((k_idx % Wn) * L, (k_idx % Wn + 1) * L)
            st["hk"][i][sl], st["hv"][i][sl] = rk, v
        tap("attn", self.r(y))
        y = self.lin(self.r(y).reshape(-1, c.dim), f"{p}.sa.o")
        xs = xs + per_frame(y, lambda t: t * ee[2][:, None])
        tap("xs_sa", xs)
        xs = xs + self.cross(i, self.r(layer_norm(xs, W[f"{p}.n3.w"], W[f"{p}.n3.b"], c.eps)), ctx_kv)
        tap("xs_ca", xs)
        if i in c.action_blocks:
            xs = self.action(i, xs, st, first, write, gm, kc, s)
        tap("xs_act", xs)
        y_in = self.r(per_frame(layer_norm(xs, eps=c.eps), lambda t: t * (1 + ee[4][:, None]) + ee[3][:, None]))
        y = self.lin(self.r(gelu_tanh(self.lin(y_in, f"{p}.ffn.0"))), f"{p}.ffn.2")
        xs = xs + per_frame(y, lambda t: t * ee[5][:, None])
        tap("xs_out", xs)
        return xs

    def head(self, xs, e):
        c, W = self.cfg, self.W
        shift, scale = W["head.mod"][0] + e, W["head.mod"][1] + e
        y = self.r(layer_norm(xs, eps=c.eps) * (1 + scale) + shift)
        return self.lin(y, "head")

    def net(self, st, x, t: float, first: bool, write: bool, inputs, ctx_kvs=None, kb_kv=None):
        """``_net`` (static.py:194-230): latent x [16, F, H, W] -> x0 (bf16-rounded latent).

        ``inputs``: dict with cc [20, F, H, W], vis [257, ctx_dim], gm [F, pad_t, 2],
        kc [kc_len, 4], k (chunk index)."""
        c = self.cfg
        s = c.frames * inputs["k"]
        fi = rope_table(c, inputs["k"], self.freqs)
        xs = self.patch_embed(x, inputs["cc"])
        e, e0 = self.time_embed(t)
        if ctx_kvs is None:
            ctx = self.context(inputs["vis"])
            ctx_kvs = [self.cross_kv(i, ctx) for i in range(c.layers)]
        for i in range(c.layers):
            xs = self.block(i, xs, e0[None].expand(c.frames, 6, c.dim), fi, st, first, write, ctx_kvs[i],
                            inputs.get("gm"), inputs.get("kc"), s)
        out = self.head(xs, e)
        flow = self.unpatchify(out)
        return self.i(x.float() - sigma_of(int(t)) * flow)

    def chunk(self, st, x_in, noise: Sequence[torch.Tensor], inputs, first: bool):
        """``_chunk`` (static.py:232-242): all denoising steps, then the context forward at t = 0.

        x_in [C, F, H, W]; ``noise[i]`` [F, C, H, W] as drawn by ``_prep`` (static.py:59,126)."""
        c = self.cfg
        ctx = self.context(inputs["vis"])
        ctx_kvs = [self.cross_kv(i, ctx) for i in range(c.layers)]
        x = self.i(x_in.float())
        n = len(c.steps)
        den = None
        for i in range(n):
            den = self.net(st, x, c.steps[i], first, False, inputs, ctx_kvs)
            if i < n - 1:
                sg = sigma_of(c.steps[i + 1])
                x = self.i((1 - sg) * den + sg * noise[i].float().transpose(0, 1))   # noise is [F, C, H, W]
        self.net(st, den, 0.0, first, True, inputs, ctx_kvs)
        return den

    def prefill(self, st, lat, inputs, first: bool):
        """``_prefill`` (static.py:244-245): one context forward over a known latent."""
        self.net(st, self.i(lat.float()), 0.0, first, True, inputs)

    def block_forward(self, xs, t: float, hist_k, hist_v, vis, k: int = 0, taps=None):
        """one block, residual tokens in, residual tokens out; keys are
        [history | current] (steady chunk k; with a window of W chunks the first min(k, W)
        slots of ``hist_k`` / ``hist_v`` are filled).  ``taps`` as in :meth:`block`."""
        c = self.cfg
        st = self.new_state()
        st["hk"][0], st["hv"][0] = hist_k, hist_v
        _, e0 = self.time_embed(t)
        ctx = self.context(vis)
        return self.block(0, xs.float(), e0[None].expand(c.frames, 6, c.dim), rope_table(c, k, self.freqs),
                          st, False, False, self.cross_kv(0, ctx), s=c.frames * k, taps=taps)
