"""FlashLatentUpsampler on the B200 conv kernel (``srdit_conv3x3``).

The reference's optional latent upsampler (video_refiner/wan/modules/
latent_upsampler/flash_latent_up.py:326-570; built by causal_inference.py:
368-410 from configs/latent_upsampler_flash.yaml and run once per clip on the
LR latent before the refinement loop, :412-424): a PixelShuffle head, a stack
of TAEHV-style memory blocks and a 3x3 projection, every layer a 3x3 conv of
bf16 frames. Here each conv is one ``srdit_conv3x3`` launch on channels-last
frames [B*T, H, W, C], with the ops that follow it fused into its epilogue:

  * head (:141-180): conv(in -> mid r^2) with the PixelShuffle(r) folded into
    the store, ReLU after the last stage;
  * memory block (:311-325): conv over torch.cat([h, past]) -- the kernel reads
    the previous frame of the clip as its second source, so the concatenation
    and the shifted ``past`` tensor (:452-476) never exist -- ReLU, conv, ReLU,
    conv + h, ReLU;
  * final projection (:386), plus the residual skip head and
    ``skip + residual_scale * correction`` when ``residual=True`` (:553-564).

Supported: any integer upsample_scale whose factors are 2, 3 or 4 per stage,
activation "relu" (the shipped config), memory_init "zero" / "replicate",
residual on or off, the parallel forward (the default, and the one the
pipeline calls). ``parallel=False`` without caches gives the same result and is
accepted; carried caches and the EMA memory (``ema_alpha``) are refused.
"""
from __future__ import annotations

import torch

from . import _lib, ops


def _head_factors(scale: int):
    """_build_upsample_head's decomposition (flash_latent_up.py:159-166)."""
    factors, rem = [], scale
    while rem % 2 == 0:
        factors.append(2)
        rem //= 2
    if rem > 1:
        factors.append(rem)
    return factors


def _pad64(c: int) -> int:
    return (c + 63) // 64 * 64


class _Conv:
    """One 3x3 conv in the kernel's layout: K-major bf16 weight, fp32 bias."""

    def __init__(self, sd, prefix, *, n_src=1, cin_pad=None, shuffle=1, device):
        w, b = sd[prefix + ".weight"], sd[prefix + ".bias"]
        self.cout = w.shape[0]
        self.cin = w.shape[1] // n_src
        self.cin_pad = cin_pad or _pad64(self.cin)
        self.n_src, self.shuffle = n_src, shuffle
        self.w = ops.conv_weight(w, n_src=n_src, cin_pad=self.cin_pad, shuffle=shuffle).to(device)
        self.b = ops.conv_bias(b, shuffle=shuffle).to(device)

    def __call__(self, x, T, **kw):
        return ops.conv3x3(x, self.w, self.b, frames_per_clip=T, n_src=self.n_src,
                           shuffle=self.shuffle, **kw)


class FlashLatentUpsampler:
    """Drop-in for the reference's ``FlashLatentUpsampler`` forward: same
    constructor arguments (weights from the reference module's ``state_dict``,
    ``sd``), ``forward(latent [B, C, T, H, W])`` -> [B, C_out, T, s H, s W] bf16."""

    def __init__(self, sd: dict, in_channels: int = 16, out_channels: int | None = None,
                 mid_channels: int = 128, num_blocks: int = 9, upsample_scale: int = 2,
                 activation: str = "relu", residual: bool = False, residual_scale: float = 1.0,
                 memory_init: str = "zero", zero_init_final: bool = True,
                 default_parallel: bool = True, ema_alpha: float | None = None,
                 init_mode: str = "nearest", device="cuda"):
        # the reference's own argument checks (flash_latent_up.py:357-363)
        if num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, got {num_blocks}.")
        if memory_init not in ("zero", "replicate"):
            raise ValueError("memory_init must be 'zero' or 'replicate'.")
        if not isinstance(upsample_scale, int) or upsample_scale < 1:
            raise ValueError(f"upsample_scale must be a positive integer, got {upsample_scale}.")
        if str(activation).lower() != "relu":
            raise _lib.SrditError(f"activation {activation!r}: the B200 path fuses ReLU only")
        if ema_alpha is not None:
            raise _lib.SrditError("the EMA memory (ema_alpha) is not supported by the B200 path")
        factors = _head_factors(upsample_scale)
        if any(f > 4 for f in factors):
            raise _lib.SrditError(f"upsample_scale {upsample_scale}: head stages up to x4 only")
        self.in_channels = in_channels
        self.out_channels = out_channels or in_channels
        self.mid_channels = mid_channels
        self.num_blocks = num_blocks
        self.upsample_scale = upsample_scale
        self.residual = residual
        self.residual_scale = float(residual_scale)
        self.memory_init = memory_init
        self.default_parallel = bool(default_parallel)
        self.device = torch.device(device)
        dev = self.device
        if mid_channels % 64:
            raise _lib.SrditError(f"mid_channels {mid_channels}: a multiple of 64 is needed")
        # pre_shuffle: [conv, PixelShuffle] per stage, then the activation
        self.head = [_Conv(sd, f"pre_shuffle.{2 * i}", shuffle=f, device=dev)
                     for i, f in enumerate(factors)]
        # each block: cat([h, past]) -> conv -> act -> conv -> act -> conv, + h, act
        self.blocks = [(_Conv(sd, f"blocks.{i}.conv.0", n_src=2, device=dev),
                        _Conv(sd, f"blocks.{i}.conv.2", device=dev),
                        _Conv(sd, f"blocks.{i}.conv.4", device=dev))
                       for i in range(num_blocks)]
        self.final = _Conv(sd, "final", device=dev)
        self.skip_up = ([_Conv(sd, f"skip_up.{2 * i}", shuffle=f, device=dev)
                         for i, f in enumerate(factors)] if residual else None)

    def _head(self, convs, x, T, act):
        for i, cv in enumerate(convs):
            x = cv(x, T, relu=act and i == len(convs) - 1)
            if i + 1 < len(convs) and x.shape[-1] % 64:
                x = torch.nn.functional.pad(x, (0, _pad64(x.shape[-1]) - x.shape[-1]))
        return x

    def forward(self, latent: torch.Tensor, parallel: bool | None = None, caches=None,
                return_caches: bool = False, detach_caches: bool = True):
        """flash_latent_up.py:530-570 (the parallel forward)."""
        if latent.ndim != 5:
            raise ValueError(f"Expected latent shape [B, C, T, H, W], got {latent.shape}.")
        if latent.shape[1] != self.in_channels:
            raise ValueError(f"Expected {self.in_channels} channels, got {latent.shape[1]}.")
        if parallel is None:
            parallel = self.default_parallel
        if caches is not None and parallel:
            raise ValueError("caches are only supported when parallel=False.")
        if caches is not None:
            raise _lib.SrditError("carried memory caches are not supported by the B200 path")
        B, C, T, H, W = latent.shape
        x = latent.to(self.device, torch.bfloat16).permute(0, 2, 3, 4, 1).reshape(B * T, H, W, C)
        cp = _pad64(C)
        x = torch.nn.functional.pad(x, (0, cp - C)) if cp != C else x.contiguous()
        rep = self.memory_init == "replicate"
        h = self._head(self.head, x, T, act=True)
        for c0, c1, c2 in self.blocks:
            t = c0(h, T, replicate=rep, relu=True)
            t = c1(t, T, relu=True)
            h = c2(t, T, residual=h, relu=True)
        skip = self._head(self.skip_up, x, T, act=False) if self.residual else None
        out = self.final(h, T, residual=skip, res_scale=self.residual_scale)
        s = self.upsample_scale
        out = out.reshape(B, T, s * H, s * W, self.out_channels).permute(0, 4, 1, 2, 3)
        out = out.contiguous()
        if return_caches:
            return out, [None] * self.num_blocks
        return out

    __call__ = forward

    def flops(self, T: int, H: int, W: int, B: int = 1) -> int:
        """Algorithmic FLOPs of one forward (2 per multiply-add, padded channels
        not counted)."""
        tot, hh, ww = 0, H, W
        for cv in self.head:
            tot += 2 * B * T * hh * ww * cv.cout * 9 * cv.cin
            hh, ww = hh * cv.shuffle, ww * cv.shuffle
        per_block = sum(2 * B * T * hh * ww * cv.cout * 9 * cv.cin * cv.n_src
                        for cv in self.blocks[0])
        tot += per_block * self.num_blocks
        tot += 2 * B * T * hh * ww * self.final.cout * 9 * self.final.cin
        if self.skip_up:
            h2, w2 = H, W
            for cv in self.skip_up:
                tot += 2 * B * T * h2 * w2 * cv.cout * 9 * cv.cin
                h2, w2 = h2 * cv.shuffle, w2 * cv.shuffle
        return tot

    @staticmethod
    def seeded_state_dict(in_channels=48, out_channels=None, mid_channels=128, num_blocks=8,
                          upsample_scale=2, residual=False, seed=0):
        """A state dict with the reference module's parameter names and shapes,
        filled with seeded random values (Kaiming-uniform-like scale), for runs
        without a checkpoint."""
        g = torch.Generator().manual_seed(seed)
        out_channels = out_channels or in_channels
        sd = {}

        def conv(name, cin, cout):
            bound = (1.0 / (cin * 9)) ** 0.5
            sd[name + ".weight"] = (torch.rand(cout, cin, 3, 3, generator=g) * 2 - 1) * bound
            sd[name + ".bias"] = (torch.rand(cout, generator=g) * 2 - 1) * bound

        factors = _head_factors(upsample_scale)
        cin = in_channels
        for i, f in enumerate(factors):
            conv(f"pre_shuffle.{2 * i}", cin, mid_channels * f * f)
            cin = mid_channels
        for i in range(num_blocks):
            conv(f"blocks.{i}.conv.0", 2 * mid_channels, mid_channels)
            conv(f"blocks.{i}.conv.2", mid_channels, mid_channels)
            conv(f"blocks.{i}.conv.4", mid_channels, mid_channels)
        conv("final", mid_channels, out_channels)
        if residual:
            cin = in_channels
            for i, f in enumerate(factors):
                conv(f"skip_up.{2 * i}", cin, out_channels * f * f)
                cin = out_channels
        return {k: v.to(torch.bfloat16) for k, v in sd.items()}
