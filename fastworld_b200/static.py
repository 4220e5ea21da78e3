"""``B200StaticMG``: the reference's ``StaticMG`` session object on the sm_100a engine.

Drop-in for ``fastworld/models/mg2/static.py:27-284``: the same public methods
(``capture``, ``gen_chunk``, ``prefill``, ``state``, ``load``, ``state_bytes``, ``_prep``,
``_chunk``, ``_prefill``, ``_state_tensors``) and the same static-buffer discipline: torch
allocates every buffer once, ``_prep`` fills the static inputs, and one launch call (or one
CUDA-graph replay) runs the whole chunk.  The chunk itself is the C ABI's ``fw_chunk``:
tcgen05 GEMMs, tcgen05 flash attention and fused elementwise kernels, no torch compute.

Differences from the reference, by design:
* constructed from a :class:`~fastworld_b200.config.DiTConfig` and a state dict (the
  official ``Model`` is not needed); images are registered with :meth:`add_image`;
* the session state lives in one contiguous device buffer (``state()`` returns a
  :class:`SessionState`, a list of views into one snapshot buffer), so save / restore is a
  single vectorised copy kernel;
* the history attention reads device-resident segment lengths, so the "first" and "steady"
  graphs differ only in which constant length table they point at.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib, graph as fw_graph
from ._lib import check, lib, ptr, stream_ptr
from .config import MG2, DiTConfig
from .prep import action_windows, device_prep_actions, path_seed, synthetic_image

_DT = {_lib.DT_BF16: torch.bfloat16, _lib.DT_F32: torch.float32, _lib.DT_I32: torch.int32, _lib.DT_U8: torch.uint8}


def pack_weights(cfg: DiTConfig, sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Map the flat state dict (``fastworld_b200.weights``) to the engine's tensor names:
    q/k/v and cross k/v are packed row-wise so each is one GEMM, block modulations are
    stacked into one [layers, 6, dim] table."""
    out: Dict[str, torch.Tensor] = {}
    for k, v in sd.items():
        if ".sa.q." in k or ".sa.k." in k or ".sa.v." in k or ".ca.k." in k or ".ca.v." in k or k.endswith(".mod") \
                and k.startswith("b"):
            continue
        out[k] = v
    out["mods"] = torch.stack([sd[f"b{i}.mod"] for i in range(cfg.layers)], 0)
    for i in range(cfg.layers):
        p = f"b{i}"
        for s in ("w", "b"):
            out[f"{p}.sa.qkv.{s}"] = torch.cat([sd[f"{p}.sa.q.{s}"], sd[f"{p}.sa.k.{s}"], sd[f"{p}.sa.v.{s}"]], 0)
            out[f"{p}.ca.kv.{s}"] = torch.cat([sd[f"{p}.ca.k.{s}"], sd[f"{p}.ca.v.{s}"]], 0)
    return out


class SessionState(list):
    """Snapshot of a session's state: views (one per state tensor, reference order) into one
    contiguous device buffer ``blob``."""

    def __init__(self, blob: torch.Tensor, views: List[torch.Tensor]):
        super().__init__(views)
        self.blob = blob


class B200StaticMG:
    """Session runtime.  ``tp_group`` (a ``torch.distributed`` process group, or ``True`` for
    the default group) shards the model over the group's ranks, one GPU each (BASELINE
    configs[4]): every rank constructs its object at the same time with the same arguments;
    ``weights`` is then either the full state dict (sharded here) or already this rank's part
    (``weights.shard_state_dict``).  Inputs, outputs and the call sequence are the same on
    every rank; the output latent is identical on all ranks."""

    def __init__(self, cfg: DiTConfig = MG2, weights: Optional[Dict[str, torch.Tensor]] = None, device="cuda",
                 seed: int = 0, tp_group=None, tp_peers: bool = True, device_prep: bool = False):
        cfg.validate()
        self.cfg = cfg
        self.device_prep = bool(device_prep)
        self.dev = torch.device(device)
        if self.dev.type != "cuda":
            raise RuntimeError("B200StaticMG runs on a CUDA device (sm_100a) only")
        self.tp_size, self.tp_rank = 1, 0
        if tp_group is not None:
            import torch.distributed as dist
            grp = None if tp_group is True else tp_group
            self.tp_size, self.tp_rank = dist.get_world_size(grp), dist.get_rank(grp)
        from .weights import shard_state_dict, synthetic_state_dict
        if weights is None:
            weights = synthetic_state_dict(cfg, seed, device=self.dev,
                                           shard=(self.tp_rank, self.tp_size) if self.tp_size > 1 else None)
        elif self.tp_size > 1 and weights[f"b0.sa.q.w"].shape[0] == cfg.dim:
            weights = shard_state_dict(cfg, weights, self.tp_rank, self.tp_size)
        packed = pack_weights(cfg, weights)
        self._ccfg = _lib.make_config(cfg, self.tp_size, self.tp_rank)
        h = ctypes.c_void_p()
        self._lib = lib()   # kept for __del__, which may run after module globals are cleared
        check(self._lib.fw_create(ctypes.byref(self._ccfg), ctypes.byref(h)), "fw_create")
        self._h = h
        if self.tp_size > 1:
            self._tp_connect(tp_group)
        self.buffers: Dict[str, torch.Tensor] = {}
        infos = []
        for i in range(lib().fw_tensor_count(h)):
            info = _lib.FwTensorInfo()
            check(lib().fw_tensor_info_at(h, i, ctypes.byref(info)), "fw_tensor_info_at")
            shape = tuple(info.shape[j] for j in range(info.ndim))
            infos.append((info.name.decode(), info.kind, _DT[info.dtype], shape, info.bytes))
        # session state: one contiguous blob, views in the reference order (static.py:280-281)
        st = [x for x in infos if x[1] == _lib.KIND_STATE]
        total = sum((b + 255) // 256 * 256 for *_, b in st)
        self._blob = torch.zeros(total, dtype=torch.uint8, device=self.dev)
        off, self._state_names = 0, []
        for name, _, dt, shape, nb in st:
            self.buffers[name] = self._blob[off:off + nb].view(dt).view(shape)
            self._state_names.append(name)
            off += (nb + 255) // 256 * 256
        for name, kind, dt, shape, nb in infos:
            if kind == _lib.KIND_STATE:
                continue
            if kind == _lib.KIND_WEIGHT:
                w = packed[name]
                if tuple(w.shape) != shape:
                    raise ValueError(f"weight {name}: shape {tuple(w.shape)} != {shape}")
                t = w.to(self.dev, torch.bfloat16).contiguous()
            else:
                t = torch.zeros(shape, dtype=dt, device=self.dev)
            self.buffers[name] = t
        for name, t in self.buffers.items():
            check(lib().fw_bind(h, name.encode(), ptr(t), t.numel() * t.element_size()), f"fw_bind({name})")
        check(lib().fw_finalize(h), "fw_finalize")
        torch.cuda.synchronize(self.dev)
        self._peer_maps = []
        if self.tp_size > 1 and tp_peers:
            self._tp_map_peers(tp_group)
        B = self.buffers
        self.hk = [B[f"hk.{i}"] for i in range(cfg.layers)]
        self.hv = [B[f"hv.{i}"] for i in range(cfg.layers)]
        self.mk = {i: B[f"mk.{i}"] for i in cfg.action_blocks}
        self.mv = {i: B[f"mv.{i}"] for i in cfg.action_blocks}
        self.kk = {i: B[f"kk.{i}"] for i in cfg.action_blocks}
        self.kv = {i: B[f"kv.{i}"] for i in cfg.action_blocks}
        self.x_in, self.cc, self.vis, self.gm, self.kc = B["x_in"], B["cc"], B["vis"], B["gm"], B["kc"]
        self.noise = [B[f"noise.{i}"] for i in range(len(cfg.steps) - 1)]
        self.lat_in, self.out, self.chunk_info, self.status = B["lat_in"], B["out"], B["chunk"], B["status"]
        self.steps = [int(t) for t in cfg.steps]
        self.images: Dict[str, Dict[str, torch.Tensor]] = {}
        self.graphs, self.cur_img = {}, None
        self._peers = set()

    def _tp_connect(self, tp_group) -> None:
        """Create the engine's NCCL communicator: the group's first rank draws the id, the
        host process group broadcasts it, every rank joins (blocking, collective)."""
        import torch.distributed as dist
        grp = None if tp_group is True else tp_group
        idbuf = ctypes.create_string_buffer(128)
        if self.tp_rank == 0:
            check(lib().fw_tp_unique_id(idbuf), "fw_tp_unique_id")
        obj = [idbuf.raw if self.tp_rank == 0 else None]
        src = dist.get_global_rank(grp, 0) if grp is not None else 0
        dist.broadcast_object_list(obj, src=src, group=grp, device=torch.device("cpu") if
                                   dist.get_backend(grp) == "gloo" else self.dev)
        with torch.cuda.device(self.dev):
            check(lib().fw_tp_init(self._h, obj[0]), "fw_tp_init")

    def _tp_map_peers(self, tp_group) -> None:
        """Map every other rank's engine workspace into this process (CUDA IPC, peer access) and
        hand the bases to the engine, which then reduces over NVLink with its own kernels
        instead of NCCL (``fw_tp_peers``)."""
        import torch.distributed as dist
        from . import migrate
        grp = None if tp_group is True else tp_group
        ws = self.buffers["workspace"]
        descs = [None] * self.tp_size
        dist.all_gather_object(descs, migrate.export_blob(ws), group=grp)
        bases = (ctypes.c_void_p * self.tp_size)()
        for j, d in enumerate(descs):
            if j == self.tp_rank:
                bases[j] = ws.data_ptr()
                continue
            pb = migrate.PeerBuffer(d, self.dev).__enter__()
            self._peer_maps.append(pb)
            bases[j] = pb.ptr
        check(lib().fw_tp_peers(self._h, bases, self.tp_size), "fw_tp_peers")
        dist.barrier(group=grp)   # every rank mapped before anyone launches

    def __del__(self):
        for pb in getattr(self, "_peer_maps", []):
            try:
                pb.__exit__(None, None, None)
            except Exception:
                pass
        self._peer_maps = []
        h, L = getattr(self, "_h", None), getattr(self, "_lib", None)
        if h is not None and h.value and L is not None:
            L.fw_destroy(h)
            self._h = None

    # ------------------------------------------------------------------ images
    def add_image(self, name: str, image: Optional[Dict[str, torch.Tensor]] = None, seed: int = 0,
                  max_chunks: int = 24) -> None:
        """Register a start image: ``cond_concat`` [1, 20, frames * max_chunks, H, W] and
        ``visual_context`` [1, 257, ctx_dim] (``Model.add_image``, model.py:53-68); a seeded
        synthetic image when ``image`` is None."""
        img = image if image is not None else synthetic_image(self.cfg, seed, max_chunks)
        self.images[name] = {k: v.to(self.dev, torch.bfloat16) for k, v in img.items()}

    # ------------------------------------------------------------------ inputs
    def _prep(self, path: Sequence, k: int, noise: bool = True) -> None:
        """Fill the static inputs for chunk k of `path` (static.py:76-127).  With
        ``device_prep`` set, one library kernel does it (``fw_prep``: no host copy, no torch
        kernel; the noise then comes from the library's counter-based generator instead of
        torch.randn, so it differs from the reference's stream); otherwise the host path
        reproduces the reference's inputs exactly."""
        if self.device_prep:
            return self._prep_device(path, k, noise)
        c = self.cfg
        img_name = path[0][0]
        img = self.images[img_name]
        if self.cur_img != img_name:
            self.vis.copy_(img["visual_context"])
            self.cur_img = img_name
        s = c.frames * k
        self.cc.copy_(img["cond_concat"][:, :, s:s + c.frames])
        kc, gm = action_windows(c, path, k)
        self.kc.copy_(kc[None], non_blocking=True)
        self.gm.copy_(gm[None], non_blocking=True)
        self.chunk_info.copy_(torch.tensor([k, s, 0, 0], dtype=torch.int32), non_blocking=True)
        if not noise:
            return
        g = torch.Generator(device=self.dev).manual_seed(path_seed(path[:k + 1]))
        self.x_in.copy_(torch.randn(self.x_in.shape, generator=g, device=self.dev, dtype=torch.bfloat16))
        for nb in self.noise:
            nb.copy_(torch.randn(nb.shape, generator=g, device=self.dev, dtype=torch.bfloat16))

    def _prep_device(self, path: Sequence, k: int, noise: bool = True) -> None:
        c = self.cfg
        img_name = path[0][0]
        img = self.images[img_name]
        if self.cur_img != img_name:
            vis = img["visual_context"]
            check(lib().fw_copy(ptr(self.vis), ptr(vis), vis.numel() * 2, stream_ptr()), "fw_copy(vis)")
            self.cur_img = img_name
        cond = img["cond_concat"]
        j_lo, acts = device_prep_actions(c, path, k)
        if len(acts) > _lib.FW_PREP_MAX_ACT:
            raise ValueError(f"action window spans {len(acts)} chunks (at most {_lib.FW_PREP_MAX_ACT})")
        a = _lib.FwPrepArgs()
        a.chunk, a.seed, a.draw_noise = k, path_seed(path[:k + 1]), int(bool(noise))
        a.cond, a.cond_frames, a.j_lo, a.n_act = ptr(cond), cond.shape[2], j_lo, len(acts)
        for j, v in enumerate(acts):
            for d, x in enumerate(v):
                a.actions[8 * j + d] = float(x)
        check(lib().fw_prep(self._h, ctypes.byref(a), stream_ptr()), "fw_prep")

    # ------------------------------------------------------------------ network
    def _chunk(self, first: bool) -> None:
        check(lib().fw_chunk(self._h, int(bool(first)), stream_ptr()), "fw_chunk")

    def _prefill(self, first: bool) -> None:
        check(lib().fw_prefill(self._h, int(bool(first)), stream_ptr()), "fw_prefill")

    def _net_step(self, step: int, first: bool, write: bool) -> None:
        """One forward from ``x_in`` (``lat_in`` for the context step) into ``out``."""
        check(lib().fw_forward(self._h, step, int(bool(first)), int(bool(write)), stream_ptr()), "fw_forward")

    # ------------------------------------------------------------------ public
    def capture(self, warmup: int = 2) -> None:
        """Record the four graphs (first | steady) x (generate | prefill) (static.py:248-252)."""
        fns = {(True, "gen"): lambda: self._chunk(True), (False, "gen"): lambda: self._chunk(False),
               (True, "pre"): lambda: self._prefill(True), (False, "pre"): lambda: self._prefill(False)}
        self.graphs = fw_graph.capture(fns, warmup=warmup, save=self.state, load=self.load)

    @torch.no_grad()
    def gen_chunk(self, path, k: int, graph: bool = True) -> torch.Tensor:
        self._prep(path, k)
        if graph:
            self.graphs[(k == 0, "gen")].replay()
        else:
            self._chunk(k == 0)
        return self.out.clone()

    @torch.no_grad()
    def prefill(self, lat: torch.Tensor, path, k: int, graph: bool = True) -> None:
        """Advance the state by chunk k whose latent is already known (one context forward)."""
        self._prep(path, k, noise=False)
        self.lat_in.copy_(lat)
        if graph:
            self.graphs[(k == 0, "pre")].replay()
        else:
            self._prefill(k == 0)

    def _reach(self, dev: torch.device) -> None:
        """Let this session's GPU read and write ``dev``'s memory (peer access, once per device)."""
        if dev == self.dev or dev.index in self._peers:
            return
        with torch.cuda.device(self.dev):
            check(lib().fw_peer_access(dev.index), f"fw_peer_access({dev})")
        self._peers.add(dev.index)

    def state(self, device=None) -> SessionState:
        """Snapshot of the history buffers: one copy kernel into a new device buffer, on this
        session's GPU or, with ``device``, in another GPU's memory (written over NVLink)."""
        dev = torch.device(device) if device is not None else self.dev
        self._reach(dev)
        blob = torch.empty(self._blob.numel(), dtype=torch.uint8, device=dev)
        with torch.cuda.device(self.dev):
            check(lib().fw_copy(ptr(blob), ptr(self._blob), self._blob.numel(), stream_ptr()), "fw_copy")
        views, off = [], 0
        for name in self._state_names:
            t = self.buffers[name]
            nb = t.numel() * t.element_size()
            views.append(blob[off:off + nb].view(t.dtype).view(t.shape))
            off += (nb + 255) // 256 * 256
        return SessionState(blob, views)

    def state_into(self, st: "SessionState") -> "SessionState":
        """Snapshot into an existing SessionState's buffer (same session shape) instead of a new
        allocation: a checkpoint pool recycles evicted checkpoints through this."""
        if not isinstance(st, SessionState) or st.blob.numel() != self._blob.numel():
            return self.state()
        self._reach(st.blob.device)
        with torch.cuda.device(self.dev):
            check(lib().fw_copy(ptr(st.blob), ptr(self._blob), self._blob.numel(), stream_ptr()), "fw_copy")
        return st

    def load(self, st) -> None:
        """Restore a snapshot into the live buffers (pointers baked into graphs stay valid)."""
        if isinstance(st, SessionState) and st.blob.numel() == self._blob.numel():
            self._reach(st.blob.device)     # a checkpoint placed on a peer GPU is read over NVLink
            with torch.cuda.device(self.dev):
                check(lib().fw_copy(ptr(self._blob), ptr(st.blob), self._blob.numel(), stream_ptr()), "fw_copy")
            return
        for d, s in zip(self._state_tensors(), st):
            s = s.to(d.device).contiguous()
            check(lib().fw_copy(ptr(d), ptr(s), d.numel() * d.element_size(), stream_ptr()), "fw_copy")

    def _state_tensors(self) -> List[torch.Tensor]:
        return self.hk + self.hv + list(self.mk.values()) + list(self.mv.values()) + list(self.kk.values()) + \
            list(self.kv.values())

    def state_bytes(self) -> int:
        return fw_graph.state_bytes(self._state_tensors())

    def set_tap(self, layer: Optional[int]) -> Optional[Dict[str, torch.Tensor]]:
        """Copy block ``layer``'s intermediates on every following forward (``fw_set_tap``);
        returns named views of the tap buffer (None clears the tap).  Residual stream fp32
        [L, dim]: ``xs_in``, ``xs_sa`` (after self-attention), ``xs_ca`` (after cross-attention),
        ``xs_act`` (after the action module), ``xs_out``; bf16 [L, heads, head_dim] of this
        rank: ``q`` and ``k`` after RMSNorm + RoPE, ``v``, ``attn`` (self-attention output)."""
        if layer is None:
            check(lib().fw_set_tap(self._h, -1, None, 0), "fw_set_tap")
            self._tap = None
            return None
        nb = lib().fw_tap_bytes(self._h)
        buf = torch.zeros(nb, dtype=torch.uint8, device=self.dev)
        check(lib().fw_set_tap(self._h, int(layer), ptr(buf), nb), "fw_set_tap")
        self._tap = buf
        c = self.cfg
        L, D, hl = c.tokens, c.dim, c.heads // self.tp_size
        xs_b, qb = L * D * 4, L * hl * c.head_dim * 2
        views = {}
        for j, name in enumerate(("xs_in", "xs_sa", "xs_ca", "xs_act", "xs_out")):
            views[name] = buf[j * xs_b:(j + 1) * xs_b].view(torch.float32).view(L, D)
        for j, name in enumerate(("q", "k", "v", "attn")):
            o = 5 * xs_b + j * qb
            views[name] = buf[o:o + qb].view(torch.bfloat16).view(L, hl, c.head_dim)
        return views

    def device_status(self) -> List[int]:
        """Device status words (0 = ok; otherwise a bounded wait gave up).  Synchronises."""
        return [int(v) for v in self.status.cpu()]
