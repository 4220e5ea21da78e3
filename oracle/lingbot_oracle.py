"""CPU oracle for the LingBot-World-v2 causal chunk runtime.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it.  The product path (``fastworld_b200.lingbot``)
runs the sm_100a kernels of ``csrc/lingbot.cu`` and fails loudly when its CUDA library is
missing.

It restates, op for op and in PyTorch fp32 on the CPU, the reference's ``StaticLingbot``
(``fastworld/models/lingbot_v2/static.py``):

* ``_consts``     per-step time embeddings and scheduler constants (``static.py:91-126``)
                  -> :meth:`LingbotOracle.time_embed` (constants from ``lingbot.flow_schedule``)
* ``set_prompt``  text embedding and every block's cross-attention K/V (``static.py:128-137``)
                  -> :meth:`LingbotOracle.set_prompt`
* ``_prep``       chunk slices of noise / condition / Plücker features, the RoPE table at the
                  chunk's absolute frame offset, the 3 renoising draws (``static.py:154-169``)
* ``_cam_emb`` / ``_cam_block`` / ``_hoist_cam``  camera branch (``static.py:188-207``)
* ``_net``        the DiT forward with the KV write at the plan's offset before attention over
                  the buffer's first ``key_len`` frames (``static.py:209-255``)
* ``_roll``       the end-of-chunk KV shift (``static.py:257-264``)
* ``_chunk``      4 forwards, x0 in fp64, renoising, the t = 0 KV refresh, the roll
                  (``static.py:266-281``)

The block internals of the un-vendored Wan model (LayerNorm eps 1e-6, RMSNorm over the full
width, GELU-tanh FFN, ``text_embedding`` = Linear, GELU-tanh, Linear; ``time_embedding`` =
Linear, SiLU, Linear; ``time_projection`` = SiLU, Linear; the camera layers are Linear, with
SiLU where ``static.py`` applies it) are the ones ``fastworld_b200.lingbot.param_specs`` names.
Interface tensors the reference keeps in bf16 (keys and values in the KV buffer, camera
scale / shift) are rounded to bf16 here too; everything else is fp32.
"""
from __future__ import annotations

from typing import Dict, List, Sequence

import torch

from oracle.mg2_oracle import apply_rope, attention, bf16, gelu_tanh, layer_norm, rms_norm, rope_freqs, sinusoid


class LingbotOracle:
    """``round_bf16=False`` keeps every tensor fp32 (the form the golden run of the reference's
    own code takes, with its bf16 buffers switched to fp32)."""

    def __init__(self, cfg, sd: Dict[str, torch.Tensor], round_bf16: bool = True):
        self.cfg = cfg
        self.rb = bf16 if round_bf16 else (lambda x: x)
        self.w = {k: v.float() for k, v in sd.items()}
        self.freqs = rope_freqs(cfg.head_dim)
        t, self.sig_x0, self.an_alpha, self.an_sigma = cfg.schedule()
        self.timesteps = t

    def lin(self, x, name, bias=True):
        y = x @ self.w[name + ".weight"].reshape(self.w[name + ".weight"].shape[0], -1).t()
        return y + self.w[name + ".bias"] if bias else y

    # ------------------------------------------------------------------ state
    def new_state(self) -> Dict[str, object]:
        c = self.cfg
        z = lambda: [torch.zeros(c.kv_tokens, c.heads, c.head_dim) for _ in range(c.layers)]   # noqa: E731
        return {"K": z(), "V": z()}

    # ------------------------------------------------------------------ constants
    def time_embed(self, t: float):
        e = self.lin(torch.nn.functional.silu(self.lin(sinusoid(self.cfg.freq_dim, t)[None], "time_embedding.0")),
                     "time_embedding.2")
        e0 = self.lin(torch.nn.functional.silu(e), "time_projection.1").view(6, self.cfg.dim)
        return e[0], e0

    def set_prompt(self, context: torch.Tensor):
        """context [n, text_dim] -> per block (K, V) [text_len, H, Dh] (zero-padded prompt)."""
        c = self.cfg
        ctx = torch.zeros(c.text_len, c.text_dim)
        ctx[:context.shape[0]] = context.float()
        emb = self.lin(gelu_tanh(self.lin(ctx, "text_embedding.0")), "text_embedding.2")
        kv = []
        for i in range(c.layers):
            p = f"blocks.{i}.cross_attn."
            k = rms_norm(self.lin(emb, p + "k"), self.w[p + "norm_k.weight"], c.eps)
            v = self.lin(emb, p + "v")
            kv.append((self.rb(k).view(c.text_len, c.heads, c.head_dim), self.rb(v).view(c.text_len, c.heads, c.head_dim)))
        self.xkv = kv

    # ------------------------------------------------------------------ chunk inputs
    def rope_table(self, k: int) -> torch.Tensor:
        c = self.cfg
        half = c.head_dim // 2
        parts = [half - 2 * (half // 3), half // 3, half // 3]
        ft, fh, fw = self.freqs.split(parts, dim=1)
        f, h, w, s = c.chunk, c.lat_h // 2, c.lat_w // 2, c.chunk * k
        tab = torch.cat([ft[s:s + f].view(f, 1, 1, -1).expand(f, h, w, -1),
                         fh[:h].view(1, h, 1, -1).expand(f, h, w, -1),
                         fw[:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1)
        return tab.reshape(f * h * w, -1)

    def patches(self, t: torch.Tensor) -> torch.Tensor:
        """[C, F, H, W] -> [F * H/2 * W/2, C * 4], features ordered (channel, dy, dx)."""
        C, F, H, W = t.shape
        return t.reshape(C, F, H // 2, 2, W // 2, 2).permute(1, 2, 4, 0, 3, 5).reshape(F * (H // 2) * (W // 2), C * 4)

    # ------------------------------------------------------------------ camera branch
    def camera(self, pl: torch.Tensor):
        """pl [cam_ch, C, h, w] -> per block (1 + scale, shift) [L, D], bf16-rounded."""
        emb = self.lin(self.patches(pl.float()), "patch_embedding_wancamctrl")
        emb = emb + self.lin(torch.nn.functional.silu(self.lin(emb, "c2ws_hidden_states_layer1")),
                             "c2ws_hidden_states_layer2")
        out = []
        for i in range(self.cfg.layers):
            p = f"blocks.{i}."
            h = self.lin(torch.nn.functional.silu(self.lin(emb, p + "cam_injector_layer1")),
                         p + "cam_injector_layer2") + emb
            # the eager module adds 1 to the bf16 scale tensor (static.py:207): bf16(1 + bf16(scale))
            out.append((self.rb(1.0 + self.rb(self.lin(h, p + "cam_scale_layer"))), self.rb(self.lin(h, p + "cam_shift_layer"))))
        return out

    # ------------------------------------------------------------------ network
    def net(self, st, x, y, step: int, woff: int, klen: int, fi, cam, head: bool = True):
        c = self.cfg
        L, D, H, Dh, Ft = c.tokens, c.dim, c.heads, c.head_dim, c.frame_tokens
        t = self.timesteps[step] if step < len(self.timesteps) else 0.0
        e, e0 = self.time_embed(t)
        xs = self.lin(self.patches(torch.cat([self.rb(x), self.rb(y)], 0)), "patch_embedding")
        for i in range(c.layers):
            p = f"blocks.{i}."
            ee = self.w[p + "modulation"][0] + e0
            yin = layer_norm(xs, eps=c.eps) * (1 + ee[1]) + ee[0]
            sa = p + "self_attn."
            q = rms_norm(self.lin(yin, sa + "q"), self.w[sa + "norm_q.weight"], c.eps).view(L, H, Dh)
            k = rms_norm(self.lin(yin, sa + "k"), self.w[sa + "norm_k.weight"], c.eps).view(L, H, Dh)
            v = self.lin(yin, sa + "v").view(L, H, Dh)
            rq, rk = apply_rope(self.rb(q), fi), apply_rope(self.rb(k), fi)
            K, V = st["K"][i], st["V"][i]
            K[woff * Ft:woff * Ft + L] = self.rb(rk)
            V[woff * Ft:woff * Ft + L] = self.rb(v)
            a = attention(rq, K[:klen * Ft], V[:klen * Ft]).reshape(L, D)
            xs = xs + self.lin(a, sa + "o") * ee[2]
            cam1, camb = cam[i]
            xs = cam1 * xs + camb
            ca = p + "cross_attn."
            xq = layer_norm(xs, self.w[p + "norm3.weight"], self.w[p + "norm3.bias"], c.eps)
            qc = rms_norm(self.lin(xq, ca + "q"), self.w[ca + "norm_q.weight"], c.eps).view(L, H, Dh)
            xk, xv = self.xkv[i]
            xs = xs + self.lin(attention(qc, xk, xv).reshape(L, D), ca + "o")
            hid = gelu_tanh(self.lin(layer_norm(xs, eps=c.eps) * (1 + ee[4]) + ee[3], p + "ffn.0"))
            xs = xs + self.lin(hid, p + "ffn.2") * ee[5]
        if not head:
            return None
        hm = self.w["head.modulation"][0] + e
        out = self.lin(layer_norm(xs, eps=c.eps) * (1 + hm[1]) + hm[0], "head.head")
        f, h, w = c.chunk, c.lat_h // 2, c.lat_w // 2
        u = out.view(f, h, w, 1, 2, 2, c.lat_ch)
        return torch.einsum("fhwpqrc->cfphqwr", u).reshape(c.lat_ch, f, c.lat_h, c.lat_w)

    def roll(self, st, roll) -> None:
        if roll is None:
            return
        src, dst, n = roll
        Ft = self.cfg.frame_tokens
        for B in (st["K"], st["V"]):
            for t in B:
                t[dst * Ft:(dst + n) * Ft] = t[src * Ft:(src + n) * Ft].clone()

    def chunk(self, st, k: int, plan, x_in, y, pl, noise: Sequence[torch.Tensor]):
        """One chunk: returns x0 [16, C, h, w] fp32.  ``noise``: the 3 renoising draws."""
        woff, klen, roll = plan
        fi = self.rope_table(k)
        cam = self.camera(pl)
        x = x_in.float()
        n = len(self.timesteps)
        x0 = None
        for i in range(n):
            flow = self.net(st, x, y, i, woff, klen, fi, cam)
            x0 = (x.double() - self.sig_x0[i] * flow.double()).float()
            if i < n - 1:
                x = self.an_alpha[i] * x0 + self.an_sigma[i] * noise[i].float()
        self.net(st, x0, y, n, woff, klen, fi, cam, head=False)
        self.roll(st, roll)
        return x0
