"""Oracle: the latent upsampler's forward on the CPU (test infrastructure only).

Restates FlashLatentUpsampler's parallel forward
(video_refiner/wan/modules/latent_upsampler/flash_latent_up.py:453-495 and
:530-570) for a bf16 model: every 3x3 conv is computed in float64 over the
bf16 values and rounded to bf16 once (its bias included), PixelShuffle and
ReLU are exact, and the residual adds round to bf16 as the reference's bf16
tensor arithmetic does:
  head        conv -> PixelShuffle(r) per stage, ReLU after the last
              (_build_upsample_head, :141-180)
  block       relu(bf16(conv3(relu(conv2(relu(conv1(cat[h, past])))))) + h)
              with past = the previous frame's h, the first frame's own h
              ("replicate") or zeros (FlashLatentMemBlock.forward :323-325,
              the past tensor of :466-492)
  final       conv (:386, :494)
  residual    bf16(skip + bf16(residual_scale * correction)) with skip the
              activation-free head of the input (:553-564)
"""
from __future__ import annotations

import torch


def round_bf16(x):
    """x rounded to bf16 (through fp32, as an fp32-accumulating conv rounds), kept
    in float64."""
    return x.to(torch.float32).to(torch.bfloat16).to(torch.float64)


def _conv(x, w, b):
    y = torch.nn.functional.conv2d(x, w.to(torch.float64), b.to(torch.float64), padding=1)
    return round_bf16(y)


def _head_factors(scale):
    factors, rem = [], scale
    while rem % 2 == 0:
        factors.append(2)
        rem //= 2
    if rem > 1:
        factors.append(rem)
    return factors


def _head(sd, prefix, x, factors, act):
    for i, f in enumerate(factors):
        x = _conv(x, sd[f"{prefix}.{2 * i}.weight"], sd[f"{prefix}.{2 * i}.bias"])
        x = torch.nn.functional.pixel_shuffle(x, f)
    return torch.relu(x) if act else x


def upsample(sd, latent, *, num_blocks, upsample_scale=2, residual=False, residual_scale=1.0,
             memory_init="zero"):
    """latent [B, C, T, H, W] (bf16 values) -> [B, C_out, T, sH, sW] float64 (bf16 values)."""
    B, C, T, H, W = latent.shape
    factors = _head_factors(upsample_scale)
    x = latent.to(torch.float64).permute(0, 2, 1, 3, 4).reshape(B * T, C, H, W)
    h = _head(sd, "pre_shuffle", x, factors, act=True)
    for i in range(num_blocks):
        _, c, hh, ww = h.shape
        hb = h.reshape(B, T, c, hh, ww)
        first = hb[:, :1] if memory_init == "replicate" else torch.zeros_like(hb[:, :1])
        past = torch.cat([first, hb[:, :-1]], dim=1).reshape(h.shape)
        p = f"blocks.{i}.conv"
        t = torch.relu(_conv(torch.cat([h, past], 1), sd[f"{p}.0.weight"], sd[f"{p}.0.bias"]))
        t = torch.relu(_conv(t, sd[f"{p}.2.weight"], sd[f"{p}.2.bias"]))
        t = _conv(t, sd[f"{p}.4.weight"], sd[f"{p}.4.bias"])
        h = torch.relu(round_bf16(t + h))
    out = _conv(h, sd["final.weight"], sd["final.bias"])
    if residual:
        skip = _head(sd, "skip_up", x, factors, act=False)
        out = round_bf16(skip + round_bf16(residual_scale * out))
    s = upsample_scale
    return out.reshape(B, T, -1, s * H, s * W).permute(0, 2, 1, 3, 4)
