"""Spatial (window-strip) partition of the SR-DiT forward: one process per GPU.

The alternative multi-GPU decomposition to tensor parallelism. Block-grid
window attention makes query windows independent, and every other op of a
block (LayerNorm-modulate, the Linears, the full-width q/k RMSNorm, RoPE,
cross attention over the text tokens, the FFN, the residuals) is per token. So
rank r of P refines the token columns [r * W/P, (r + 1) * W/P) of the latent
token grid -- a strip of whole query windows -- with the full model:

  * it embeds its strip of the latent (patch columns of the strip only),
  * runs every block on its 3 x h x W/P tokens, with RoPE at the strip's true
    width positions (``rope_w0``), its own KV-cache ring of the strip's
    tokens, and the window plan of the strip (the global plan's windows that
    lie in it, since the strip starts on a window boundary),
  * and the refined strips are all-gathered once per forward into the full
    latent on every rank (2.6 MB at 2K, one collective).

With windows of radius 0 along w (BASELINE's literal 3x8x8 windows) a window's
keys lie in its own strip, so nothing else crosses GPUs: weak-per-token work
with no data-path collective inside the forward. Windows that see neighbouring
columns (radius > 0 along w, the shipped 4x4 radius-3 geometry) would need a
K/V halo of radius x block-width columns per side from the neighbour strips
every block; that exchange is not built here, and such a configuration is
refused. The reference itself does not shard the refiner.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .model import SRDiT, SRDiTConfig


class SpatialSRDiT(SRDiT):
    """``SRDiT`` refining this rank's strip of token columns; ``forward_chunk``
    takes and returns the full latent (every rank gets the full refined latent).
    """

    def __init__(self, cfg: SRDiTConfig, sd: dict, device="cuda", group=None):
        initialized = dist.is_available() and dist.is_initialized()
        self.group = group
        self.world = dist.get_world_size(group) if initialized else 1
        self.rank = dist.get_rank(group) if initialized else 0
        if self.world > 1 and cfg.block_radius_hw[1] != 0:
            raise _lib.SrditError(
                "the spatial partition needs windows of radius 0 along w (no K/V halo "
                f"exchange is built); got block_radius_hw={cfg.block_radius_hw}")
        super().__init__(cfg, sd, device)

    def strip(self, W: int):
        """Token columns [w0, w1) of this rank for a grid W tokens wide."""
        P, bw = self.world, self.cfg.block_hw[1]
        if W % (P * bw):
            raise _lib.SrditError(f"{P} strips of whole {bw}-wide windows do not tile a "
                                  f"{W}-token-wide grid")
        wl = W // P
        return self.rank * wl, (self.rank + 1) * wl

    def new_cache(self, frame_tokens):
        """K/V ring of this rank's strip (``frame_tokens``: tokens of a full frame)."""
        return super().new_cache(frame_tokens // self.world)

    def _scratch_cache(self, L):
        # L here is already the strip's tokens per frame
        key = ("scratch_cache", L)
        if key not in self._bufs:
            self._bufs[key] = SRDiT.new_cache(self, L)
        return self._bufs[key]

    def forward_chunk(self, latent, t, context, **kw):
        """``SRDiT.forward_chunk`` of the full latent [C, f, H, W] on this rank's
        strip; returns the full refined latent (``return_kv``: the strip's K/V)."""
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
