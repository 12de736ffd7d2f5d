"""Spatial (window-strip) partition of the SR-DiT forward: one process per GPU.

The alternative multi-GPU decomposition to tensor parallelism. Block-grid
window attention makes query windows independent, and every other op of a
block (LayerNorm-modulate, the Linears, the full-width q/k RMSNorm, RoPE,
cross attention over the text tokens, the FFN, the residuals) is per token. So
rank r of P refines the token columns [r * W/P, (r + 1) * W/P) of the latent
token grid -- a strip of whole query windows -- with the full model:

  * it embeds its strip of the latent (patch columns of the strip only),
  * runs every block on its 3 x h x W/P tokens, with RoPE at the strip's true
    width positions (``rope_w0``) and the global window plan's rows of the
    strip's windows (``blockgrid.strip_rows``),
  * keeps a K/V ring of the strip's columns plus a halo of R = radius_w x
    block_w columns on each side that has a neighbour -- the columns its
    windows see beyond its edges (none for radius 0 along w),
  * and the refined strips are all-gathered once per forward into the full
    latent on every rank (2.6 MB at 2K, one collective).

The halo is the only data that crosses GPUs inside the forward. Every block,
the kernel that writes the chunk's roped K and V rows into the ring
(``srdit_rms_rope``) also stores the strip's R edge columns straight into the
neighbours' rings over NVLink (``halo="peer"``: plain peer stores into a ring
mapped with CUDA IPC, then a release-add of a counter in the neighbour's
memory); before its attention, each rank waits (bounded) for its neighbours'
counters. ``halo="collective"`` exchanges the same columns with
torch.distributed point-to-point calls instead (any backend; the CPU tests use
it over gloo).

Ordering of the peer stores: a rank writes its neighbour's block-i ring in
forward n + 1 only after it passed the wait of block i - 1 in that forward (of
the last block in forward n, for block 0) -- the neighbour had then written
that block's K/V, so it had finished everything before, its block-i attention
of forward n included. Each forward starts from zeroed counters: a rank zeroes
its own, then a one-element all-reduce is the barrier after which peers signal
again (every signal of the previous forward was waited for inside it), which
also keeps a captured CUDA graph of the forward valid on replay.

Strips must be at least R columns wide (the halo comes from the adjacent strips
only). The reference itself does not shard the refiner.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib, blockgrid
from .model import KVRing, SRDiT, SRDiTConfig


class HaloRing(KVRing):
    """The K/V frame rings of a strip and its halo: frames of grid_h x ext_w
    tokens, every layer's K and V in one allocation ``buf`` [2, layers, cap *
    grid_h * ext_w, dim] (one CUDA IPC mapping per neighbour), the strip's own
    columns at [col0, col0 + strip_w) of each frame row."""

    def __init__(self, layers, grid_h, ext_w, col0, strip_w, dim, kv_len, chunk, device):
        self.cap = kv_len + chunk
        self.kv_len = kv_len
        self.grid_h, self.ext_w, self.col0, self.strip_w = grid_h, ext_w, col0, strip_w
        self.frame_tokens = grid_h * ext_w
        self.buf = torch.zeros(2, layers, self.cap * self.frame_tokens, dim, dtype=torch.bfloat16,
                               device=device)
        self.k = [self.buf[0, i] for i in range(layers)]
        self.v = [self.buf[1, i] for i in range(layers)]
        self.halo = None    # per layer: _lib.RopeHalo of the neighbours' rings (peer mode)
        self.start = 0
        self.frames = 0


class SpatialSRDiT(SRDiT):
    """``SRDiT`` refining this rank's strip of token columns; ``forward_chunk``
    takes and returns the full latent (every rank gets the full refined latent).
    ``halo``: "peer" (the ring write stores the neighbours' halo columns over
    NVLink) or "collective" (torch.distributed send / recv of the columns).
    """

    def __init__(self, cfg: SRDiTConfig, sd: dict, device="cuda", group=None, halo="peer"):
        initialized = dist.is_available() and dist.is_initialized()
        self.group = group
        self.world = dist.get_world_size(group) if initialized else 1
        self.rank = dist.get_rank(group) if initialized else 0
        if halo not in ("peer", "collective"):
            raise ValueError(f"halo must be 'peer' or 'collective', not {halo!r}")
        self.halo = halo
        # halo columns per side: the windows' reach along w beyond their own block
        self.R = cfg.block_radius_hw[1] * cfg.block_hw[1] if self.world > 1 else 0
        super().__init__(cfg, sd, device)
        self._strip_plans = {}
        self._peer_bases = []   # neighbours' mapped allocations
        self._flags = None      # halo counters of this rank, one per source rank (peer mode)

    # ---- geometry
    def strip(self, W: int):
        """Token columns [w0, w1) of this rank for a grid W tokens wide."""
        return self._strip_of(self.rank, W)

    def _strip_of(self, r, W):
        P, bw = self.world, self.cfg.block_hw[1]
        if W % (P * bw):
            raise _lib.SrditError(f"{P} strips of whole {bw}-wide windows do not tile a "
                                  f"{W}-token-wide grid")
        wl = W // P
        if wl < self.R:
            raise _lib.SrditError(
                f"strips of {wl} columns are narrower than the {self.R}-column K/V halo "
                f"(block_radius_hw={self.cfg.block_radius_hw}, block_hw={self.cfg.block_hw}): "
                f"use fewer ranks")
        return r * wl, (r + 1) * wl

    def _ext_of(self, r, W):
        """Columns [e0, e1) of rank r's K/V frames: its strip and its halo."""
        w0, w1 = self._strip_of(r, W)
        return max(0, w0 - self.R), min(W, w1 + self.R)

    def _kv_width(self, w):
        if self.world == 1:
            return w
        e0, e1 = self._ext_of(self.rank, w * self.world)
        return e1 - e0

    def _window_plan(self, f, f_kv, h, w, streaming, mode, independent_frames):
        """The rows of the full grid's plan whose windows lie in this strip, in the
        strip's query and K/V column coordinates."""
        if self.world == 1:
            return super()._window_plan(f, f_kv, h, w, streaming, mode, independent_frames)
        W = w * self.world
        key = (f, f_kv, h, W, streaming, mode, independent_frames)
        plan = self._strip_plans.get(key)
        if plan is None:
            full = super()._window_plan(f, f_kv, h, W, streaming, mode, independent_frames)
            stride = int(full["p_stride"])
            w0, w1 = self.strip(W)
            e0, e1 = self._ext_of(self.rank, W)
            rows = blockgrid.strip_rows(torch.as_tensor(full["params"]), stride, w0, w1, e0,
                                        e1 - e0)
            plan = self._strip_plans[key] = {
                "params": rows, "n_w": rows.shape[0], "p_stride": stride,
                "hr_base": f * h * (e1 - e0) if mode is not None else 0}
        return plan

    # ---- rings
    def new_cache(self, frame_tokens, grid_hw=None):
        """K/V ring of this rank's strip and halo (``frame_tokens``: tokens of a full
        frame; ``grid_hw``: its (h, W) token grid, needed when there is a halo).
        A collective step with a halo in peer mode: every rank must reach it."""
        if not self.R:
            return super().new_cache(frame_tokens // self.world)
        if grid_hw is None or grid_hw[0] * grid_hw[1] != frame_tokens:
            raise _lib.SrditError("a strip with a K/V halo needs the frame's token grid "
                                  "(new_cache(h * W, grid_hw=(h, W)))")
        return self._halo_ring(*grid_hw)

    def _scratch_cache(self, L, grid_hw=None):
        # L / grid_hw: the strip's tokens per frame and its (h, w)
        if not self.R:
            key = ("scratch_cache", L)
            if key not in self._bufs:
                self._bufs[key] = SRDiT.new_cache(self, L)
            return self._bufs[key]
        h, wl = grid_hw
        key = ("scratch_halo", h, wl)
        if key not in self._bufs:
            self._bufs[key] = self._halo_ring(h, wl * self.world)
        return self._bufs[key]

    def _halo_ring(self, h, W):
        c = self.cfg
        w0, w1 = self.strip(W)
        e0, e1 = self._ext_of(self.rank, W)
        ring = HaloRing(c.num_layers, h, e1 - e0, w0 - e0, w1 - w0, self.kv_width, c.kv_len,
                        c.chunk_frames, self.device)
        if self.halo == "peer":
            self._link(ring, h, W)
        return ring

    def _neighbours(self):
        """[(side, rank)] of the adjacent strips: side 0 left, 1 right."""
        out = []
        if self.rank > 0:
            out.append((0, self.rank - 1))
        if self.rank < self.world - 1:
            out.append((1, self.rank + 1))
        return out

    def _share(self, t):
        """Base addresses of every rank's ``t`` in this process (None for ranks
        that are not neighbours): a collective step."""
        ops = self.ops
        handle, offset = ops.ipc_handle(t)
        allh = [None] * self.world
        dist.all_gather_object(allh, (handle, offset), group=self.group)
        addrs = [None] * self.world
        addrs[self.rank] = t.data_ptr()
        for _, n in self._neighbours():
            base = ops.ipc_open(allh[n][0])
            self._peer_bases.append(base)
            addrs[n] = base + allh[n][1]
        return addrs

    def _link(self, ring, h, W):
        """Map the neighbours' rings of the same grid and build each layer's
        ``RopeHalo``: this strip's first R columns go to the left neighbour, its
        last R to the right one, at their places in the neighbours' frames."""
        import ctypes
        if self._flags is None:
            dev = self.device
            self._flags = torch.zeros(_lib.SRDIT_MAX_RANKS, dtype=torch.int32, device=dev)
            self._done = torch.zeros(1, dtype=torch.int32, device=dev)
            self._bar = torch.zeros(1, dtype=torch.float32, device=dev)
            self._flag_addrs = self._share(self._flags)
            self._mask = sum(1 << n for _, n in self._neighbours())
        addrs = self._share(ring.buf)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)   # every ring mapped and zeroed before the first store
        w0, w1 = self.strip(W)
        wl, R, D = w1 - w0, self.R, self.kv_width
        layers = self.cfg.num_layers
        ring.halo = []
        for li in range(layers):
            hs = _lib.RopeHalo()
            for side, n in self._neighbours():
                n_e0, n_e1 = self._ext_of(n, W)
                layer_bytes = ring.cap * h * (n_e1 - n_e0) * D * 2
                hs.k[side] = addrs[n] + li * layer_bytes
                hs.v[side] = addrs[n] + (layers + li) * layer_bytes
                hs.grid_w[side] = n_e1 - n_e0
                hs.w0[side] = w0 - n_e0
                hs.col_lo[side], hs.col_hi[side] = (0, R) if side == 0 else (wl - R, wl)
                hs.flag[side] = self._flag_addrs[n] + 4 * self.rank
            hs.done = ctypes.c_void_p(self._done.data_ptr()).value
            ring.halo.append(hs)

    # ---- per-forward hooks
    def _begin_forward(self):
        if self.R and self.halo == "peer":
            self._flags.zero_()
            dist.all_reduce(self._bar, group=self.group)

    def _ring_kw(self, li, cache, w):
        if not self.R:
            return {}
        return dict(dst_grid_w=cache.ext_w, dst_w0=cache.col0,
                    halo=cache.halo[li] if cache.halo is not None else None)

    def _kv_sync(self, li, cache, slot_cur, f):
        if not self.R:
            return
        if self.halo == "peer":
            self.ops.wait_counters(self._flags.data_ptr(), self._mask, li + 1,
                                   status=self.status, device=self.device)
        else:
            self._exchange(li, cache, slot_cur, f)

    def _exchange(self, li, cache, slot_cur, f):
        """torch.distributed exchange of block ``li``'s halo columns of the chunk's
        frames with the adjacent strips (``halo="collective"``)."""
        h, E, c0, wl, R = cache.grid_h, cache.ext_w, cache.col0, cache.strip_w, self.R
        slots = [(slot_cur + j) % cache.cap for j in range(f)]
        views = [t.view(cache.cap, h, E, -1) for t in (cache.k[li], cache.v[li])]
        p2p, recvs = [], []
        for side, n in self._neighbours():
            send_c = (c0, c0 + R) if side == 0 else (c0 + wl - R, c0 + wl)
            recv_c = (c0 - R, c0) if side == 0 else (c0 + wl, c0 + wl + R)
            send = torch.stack([torch.stack([v[s, :, send_c[0]:send_c[1]] for s in slots])
                                for v in views]).contiguous()
            recv = torch.empty_like(send)
            peer = n if self.group is None else dist.get_global_rank(self.group, n)
            p2p += [dist.P2POp(dist.isend, send, peer, self.group),
                    dist.P2POp(dist.irecv, recv, peer, self.group)]
            recvs.append((recv, recv_c))
        for req in dist.batch_isend_irecv(p2p):
            req.wait()
        for recv, (a, b) in recvs:
            for i, v in enumerate(views):
                for j, s in enumerate(slots):
                    v[s, :, a:b] = recv[i, j]

    # ---- forward
    def forward_chunk(self, latent, t, context, **kw):
        """``SRDiT.forward_chunk`` of the full latent [C, f, H, W] on this rank's
        strip; returns the full refined latent (``return_kv``: the strip's K/V,
        halo columns included)."""
        pw = self.cfg.patch_size[2]
        W = latent.shape[-1] // pw
        w0, w1 = self.strip(W)
        self.rope_w0 = w0
        local = latent[..., w0 * pw:w1 * pw].contiguous()
        res = super().forward_chunk(local, t, context, **kw)
        if res is None or self.world == 1:
            return res
        if kw.get("return_kv"):
            out, kv = res
            return self._gather(out), kv
        return self._gather(res)

    def _gather(self, out):
        """All-gather the strips [C, f, H, W/P] along the width."""
        parts = [torch.empty_like(out) for _ in range(self.world)]
        dist.all_gather(parts, out.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    def close(self):
        """Unmap the neighbours' allocations."""
        for b in self._peer_bases:
            self.ops.ipc_close(b)
        self._peer_bases = []
