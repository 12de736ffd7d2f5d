"""Oracle: the SR-DiT streaming forward for one sample (test infrastructure only).

Restates ``WanModel._forward_inference`` (video_refiner/wan/modules/sr_dit/models.py:
1877-2002) with ``_prepare_embeddings`` (:1827-1875), the blocks of
``oracle.block`` and ``Head`` + ``unpatchify`` (:1357-1384, :2234-2257), on the
CPU. The time embedding and head run in fp32 (the reference runs them under a
CUDA fp32 autocast, which is a no-op on the CPU), everything else in bf16.
"""
from __future__ import annotations

import torch

from . import block as oblock
from . import numerics as onum


def sinusoidal(dim, position):
    """models.py:66-77."""
    half = dim // 2
    position = position.to(torch.float64)
    s = torch.outer(position, torch.pow(10000, -torch.arange(half).to(position).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


def forward_chunk(sd, cfg, latent, t, context, *, caches=None, t_offset=0, kv_len=9,
                  linear="fp8", fp8caches=None, anchor=None, anchor_align="frame",
                  block_outputs=None):
    """Returns (out [C_out, f, H, W] bf16, new per-layer caches [(K, V)]).
    ``block_outputs`` (a list, optional) receives every block's output [L, dim]."""
    bf = lambda n: sd[n].to(torch.bfloat16)  # noqa: E731
    f32 = lambda n: sd[n].float()  # noqa: E731
    D = cfg.dim
    x = torch.nn.functional.conv3d(latent[None].to(torch.bfloat16), bf("patch_embedding.weight"),
                                   bf("patch_embedding.bias"), stride=cfg.patch_size)
    f, h, w = (int(v) for v in x.shape[2:])
    x = x.flatten(2).transpose(1, 2)[0]
    e = sinusoidal(cfg.freq_dim, torch.tensor([float(t)])).float()
    e = torch.nn.functional.linear(e, f32("time_embedding.0.weight"), f32("time_embedding.0.bias"))
    e = torch.nn.functional.linear(torch.nn.functional.silu(e), f32("time_embedding.2.weight"),
                                   f32("time_embedding.2.bias"))
    e0 = torch.nn.functional.linear(torch.nn.functional.silu(e), f32("time_projection.1.weight"),
                                    f32("time_projection.1.bias")).view(6, D)
    ctx = context.to(torch.bfloat16)
    if ctx.shape[0] < cfg.text_len:
        ctx = torch.cat([ctx, ctx.new_zeros(cfg.text_len - ctx.shape[0], ctx.shape[1])])
    ctx = torch.nn.functional.linear(ctx, bf("text_embedding.0.weight"), bf("text_embedding.0.bias"))
    ctx = torch.nn.functional.gelu(ctx, approximate="tanh")
    ctx = torch.nn.functional.linear(ctx, bf("text_embedding.2.weight"), bf("text_embedding.2.bias"))
    head_dim = D // cfg.num_heads
    td, hd, wd = onum.rope_axis_dims(head_dim)
    freqs = torch.cat([onum.rope_params(cfg.rope_rows, td), onum.rope_params(cfg.rope_rows, hd),
                       onum.rope_params(cfg.rope_rows, wd)], dim=1)
    new = []
    fp8caches = fp8caches if fp8caches is not None else [dict() for _ in range(cfg.num_layers)]
    for i in range(cfg.num_layers):
        pre = f"blocks.{i}."
        wts = {k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)}
        wts = {k: (v.float() if k == "modulation" else v.to(torch.bfloat16)) for k, v in wts.items()}
        ck, cv = (caches[i] if caches is not None else (None, None))
        ak, av = (anchor[i] if anchor is not None else (None, None))
        x, nk, nv = oblock.block_forward(
            wts, x, e0, ctx, grid=(f, h, w), freqs=freqs, t_offset=t_offset, cache_k=ck,
            cache_v=cv, kv_len=kv_len, anchor_k=ak, anchor_v=av, anchor_align=anchor_align,
            block_hw=cfg.block_hw, radius_hw=cfg.block_radius_hw,
            block_t=cfg.block_t, heads=cfg.num_heads, eps=cfg.eps, linear=linear,
            fp8cache=fp8caches[i])
        new.append((nk, nv))
        if block_outputs is not None:
            block_outputs.append(x)
    mod = f32("head.modulation").reshape(2, D) + e
    n = onum.layer_norm(x, cfg.eps)
    y = torch.nn.functional.linear(n.float() * (1 + mod[1]) + mod[0], f32("head.head.weight"),
                                   f32("head.head.bias"))
    p = cfg.patch_size
    y = y.view(f, h, w, *p, cfg.out_dim)
    y = torch.einsum("fhwpqrc->cfphqwr", y).reshape(cfg.out_dim, f * p[0], h * p[1], w * p[2])
    return y.to(torch.bfloat16), new
