"""Oracle: one SR-DiT block, streaming inference branch (test infrastructure only).

Restates ``WanAttentionBlock.forward`` (video_refiner/wan/modules/sr_dit/models.py:
1207-1354, the non-teacher-forcing branch :1304-1351) with the window
self-attention path of ``WanSelfAttention.forward`` (models.py:583-676) and the
cross-attention of ``WanT2VCrossAttention.forward`` (models.py:1042-1062), in
torch on the CPU, with the reference's dtype / rounding points:

  e        = modulation + e0                                    fp32   (:1305-1306)
  attn_in  = bf16( bf16(LN(x)) * (1 + e1) + e0 )                       (:1308-1312)
  q, k, v  = Linear(attn_in); q, k = RMSNorm(3072); RoPE (fp64)        (:602-626)
  y        = o( window_attention(q, k, v | cache, anchor) )            (:651-673)
  x        = bf16( x + y * e2 )                                 fp32   (:1349-1351)
  x        = x + cross_o( attn( norm3(x) ) )                    bf16   (:1257)
  x        = bf16( x + ffn( bf16( bf16(LN(x)) * (1 + e4) + e3 ) ) * e5 )  (:1258-1262)

``linear`` selects the Linear semantics: "bf16" (nn.Linear in bf16, pinned
against the reference's own CPU output in tests/golden/block.npz) or "fp8"
(the Fp8Linear restatement of oracle.numerics.fp8_linear).
"""
from __future__ import annotations

import torch

from . import blockgrid as obg
from . import numerics as onum
from . import winattn as owa


def _lin(x, wts, name, linear, fp8cache):
    w = wts[f"{name}.weight"]
    b = wts.get(f"{name}.bias")
    if linear == "bf16":
        return torch.nn.functional.linear(x, w, b)
    if name not in fp8cache:
        fp8cache[name] = onum.fp8_linear_weights(w)
    wq, ws = fp8cache[name]
    return onum.fp8_linear(x, wq, ws, b)


def block_forward(wts, x, e0, ctx, *, grid, freqs, t_offset, cache_k=None, cache_v=None,
                  kv_len=None, anchor_k=None, anchor_v=None, anchor_align="frame",
                  block_hw=(4, 4), radius_hw=(3, 3), block_t=3, heads, eps=1e-6,
                  linear="bf16", fp8cache=None):
    """x [L, dim] bf16, e0 [6, dim] fp32, ctx [Lc, dim] bf16 (already text-embedded).

    Returns (x_out bf16 [L, dim], new_cache_k, new_cache_v) with caches
    [frames*h*w, heads, d] (roped K / raw V), truncated to kv_len frames.
    """
    fp8cache = {} if fp8cache is None else fp8cache
    f, h, w = grid
    Ltok, dim = x.shape
    d = dim // heads
    e = (wts["modulation"].float().reshape(6, dim) + e0.float())
    ln = onum.layer_norm(x, eps)
    attn_in = (ln.float() * (1 + e[1]) + e[0]).to(torch.bfloat16)
    q = onum.rms_norm(_lin(attn_in, wts, "self_attn.q", linear, fp8cache), wts["self_attn.norm_q.weight"], eps)
    k = onum.rms_norm(_lin(attn_in, wts, "self_attn.k", linear, fp8cache), wts["self_attn.norm_k.weight"], eps)
    v = _lin(attn_in, wts, "self_attn.v", linear, fp8cache)
    q = onum.rope_apply(q.view(Ltok, heads, d), grid, freqs, t_offset).to(torch.bfloat16)
    k = onum.rope_apply(k.view(Ltok, heads, d), grid, freqs, t_offset).to(torch.bfloat16)
    v = v.view(Ltok, heads, d)
    if cache_k is not None:
        full_k = torch.cat([cache_k, k])
        full_v = torch.cat([cache_v, v])
    else:
        full_k, full_v = k, v
    L = h * w
    f_kv = full_k.shape[0] // L
    streaming = cache_k is not None or anchor_k is not None
    spec = obg.make_spec(f, f_kv, h, w, block_t=block_t, block_hw=block_hw,
                         block_radius_hw=radius_hw, streaming=streaming)
    mode = None if anchor_k is None else anchor_align
    plan = obg.build_plan(spec, mode)
    kx, vx = full_k, full_v
    if anchor_k is not None:
        kx = torch.cat([anchor_k, full_k])
        vx = torch.cat([anchor_v, full_v])
    att = owa.run_plan(q, kx, vx, plan, f_cur=f, h=h, w=w, dtype=torch.float32)
    att = att.to(torch.bfloat16).reshape(Ltok, dim)
    y = _lin(att, wts, "self_attn.o", linear, fp8cache)
    x = (x.float() + y.float() * e[2]).to(torch.bfloat16)
    # cross attention (norm3 affine LN; no RoPE; dense over the text tokens)
    xn = onum.layer_norm(x, eps, wts["norm3.weight"], wts["norm3.bias"])
    cq = onum.rms_norm(_lin(xn, wts, "cross_attn.q", linear, fp8cache), wts["cross_attn.norm_q.weight"], eps)
    ck = onum.rms_norm(_lin(ctx, wts, "cross_attn.k", linear, fp8cache), wts["cross_attn.norm_k.weight"], eps)
    cv = _lin(ctx, wts, "cross_attn.v", linear, fp8cache)
    qh = cq.view(Ltok, heads, d).transpose(0, 1).float()
    kh = ck.view(-1, heads, d).transpose(0, 1).float()
    vh = cv.view(-1, heads, d).transpose(0, 1).float()
    p = torch.softmax(qh @ kh.transpose(1, 2) * d ** -0.5, dim=-1)
    co = (p @ vh).transpose(0, 1).reshape(Ltok, dim).to(torch.bfloat16)
    x = x + _lin(co, wts, "cross_attn.o", linear, fp8cache)
    # FFN
    ln2 = onum.layer_norm(x, eps)
    ffn_in = (ln2.float() * (1 + e[4]) + e[3]).to(torch.bfloat16)
    hdn = onum.gelu_tanh(_lin(ffn_in, wts, "ffn.0", linear, fp8cache))
    y = _lin(hdn, wts, "ffn.2", linear, fp8cache)
    x = (x.float() + y.float() * e[5]).to(torch.bfloat16)
    if kv_len is not None and f_kv > kv_len:
        full_k, full_v = full_k[-kv_len * L:], full_v[-kv_len * L:]
    return x, full_k, full_v
