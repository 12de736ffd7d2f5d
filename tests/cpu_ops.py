"""A CPU stand-in for the kernel launchers of ``dreamx-creator_b200.ops`` -- TEST DOUBLE.

Same function names and arguments as the CUDA wrappers, computed with torch on
the CPU (the oracle's numerics). The CPU tests substitute it for a model's
``ops`` table to run the host-side orchestration -- weight sharding, the
sequence split, where each collective sits -- under the gloo backend without a
GPU. It is never the product path: the model refuses to build without CUDA
unless a test swaps its table, and only tests import this module.
"""
from __future__ import annotations

import torch

from oracle import numerics as onum
from oracle import winattn as owa

BF16 = torch.bfloat16
FP8_MAX = 448.0


def quant_rowwise(x, amax=None, q=None, scale=None):
    xf = x.float()
    a = amax if amax is not None else xf.abs().amax(-1)
    s = (a / FP8_MAX).clamp_min(1e-12)
    qq = (xf / s[:, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    if q is None:
        q = torch.empty_like(qq)
    if scale is None:
        scale = torch.empty_like(s)
    q.copy_(qq)
    scale.copy_(s)
    return q, scale


def ln_mod_quant(x, eps=1e-6, *, ln_weight=None, ln_bias=None, shift=None, scale=None, q=None,
                 qscale=None):
    n = onum.layer_norm(x, eps, ln_weight, ln_bias)
    if scale is not None:
        n = (n.float() * (1 + scale) + shift).to(BF16)
    return quant_rowwise(n, q=q, scale=qscale)


def fp8_gemm(a_fp8, a_scale, w_fp8, w_scale, bias=None, out=None, *, epilogue="store",
             residual=None, gate=None, row_amax=None, status=None, v_ring=None):
    if v_ring is not None:   # columns [col0, N) into the frame ring, the rest into out
        ring, col0, ft, slot0, n_slots = v_ring
        full = fp8_gemm(a_fp8, a_scale, w_fp8, w_scale, bias)
        out[:, :col0].copy_(full[:, :col0])
        rows = torch.arange(full.shape[0])
        f, sp = rows // ft, rows % ft
        ring[((slot0 + f) % n_slots) * ft + sp] = full[:, col0:]
        return out
    y = (a_fp8.double() @ w_fp8.double().t()) * a_scale.double()[:, None] * w_scale.double()
    if bias is not None:
        y = y + bias.double()
    yb = y.to(BF16)
    if epilogue == "store":
        res = yb
    elif epilogue == "gelu":
        res = onum.gelu_tanh(yb)
        row_amax.copy_(torch.maximum(row_amax, res.float().abs().amax(-1)))
    elif epilogue == "gated_res":
        res = (residual.float() + yb.float() * gate).to(BF16)
    else:
        res = (residual.float() + yb.float()).to(BF16)
    if out is None:
        return res
    out.copy_(res)
    return out


def row_reduce(x, op, out=None):
    xf = x.float()
    r = xf.pow(2).sum(-1) if op == "sumsq" else xf.abs().amax(-1)
    if out is None:
        return r
    out.copy_(r)
    return out


def residual(x, parts, bias=None, gate=None):
    p3 = parts if parts.dim() == 3 else parts.unsqueeze(0)
    y = p3.float().sum(0)
    if bias is not None:
        y = y + bias.float()
    y = y.to(BF16).float()
    x.copy_(((x.float() + y * gate) if gate is not None else (x.float() + y)).to(BF16))
    return x


def rms_rope(src, weight, eps, dst, *, frame_tokens, slot0=0, n_slots=1 << 30, cos=None,
             sin=None, grid_h=0, grid_w=0, t_offset=0, v_src=None, v_dst=None, ss=None,
             norm_width=0, t_offset_dev=None, w_offset=0, dst_grid_w=0, dst_w0=0, halo=None):
    if halo is not None:
        raise NotImplementedError("the CPU double has no peer memory")
    M, K = src.shape
    if t_offset_dev is not None:
        t_offset = t_offset + int(t_offset_dev[0])
    xf = src.float()
    if ss is not None:
        r = torch.rsqrt(ss / norm_width + eps)
    else:
        r = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    o = (xf * r[:, None]).to(BF16) * weight
    rows = torch.arange(M)
    f, sp = rows // frame_tokens, rows % frame_tokens
    if cos is not None:
        d = torch.arange(K // 2) % 64
        pos = torch.where(d[None] < 22, (t_offset + f)[:, None],
                          torch.where(d[None] < 43, (sp // grid_w)[:, None],
                                      (sp % grid_w + w_offset)[:, None]))
        c, s = cos[pos, d[None]], sin[pos, d[None]]
        x2 = o.double().view(M, K // 2, 2)
        o = torch.stack([x2[..., 0] * c - x2[..., 1] * s, x2[..., 0] * s + x2[..., 1] * c],
                        -1).view(M, K).to(BF16)
    if dst_grid_w:
        drow = (((slot0 + f) % n_slots) * grid_h + sp // grid_w) * dst_grid_w + sp % grid_w + dst_w0
    else:
        drow = ((slot0 + f) % n_slots) * frame_tokens + sp
    res = o.clone()
    dst[drow] = res
    if v_src is not None:
        v_dst[drow] = v_src.clone()
    return dst


def winattn(q, k_hr, v_hr, out, *, params_dev, n_w, p_stride, anchor_mode, geom, tiling,
            k_anchor=None, v_anchor=None, status=None, flops=0):
    n = geom.n_heads
    scale = geom.scale
    if geom.q_frames == 1 and geom.kv_slots == 1:
        # dense attention over every key (the cross-attention "window"; a
        # self-attention ring has at least two slots)
        qh = q.double().view(q.shape[0], n, 128)
        kh = k_hr.double().reshape(k_hr.shape[0], n, 128)
        vh = v_hr.double().reshape(v_hr.shape[0], n, 128)
        att = torch.softmax(torch.einsum("qnd,knd->nqk", qh, kh) * scale, -1)
        out.copy_(torch.einsum("nqk,knd->qnd", att, vh).reshape(out.shape).to(BF16))
        return out
    f, h, w = geom.q_frames, geom.q_h, geom.q_w
    L = geom.kv_h * geom.kv_w
    params = params_dev.cpu()
    if geom.col_split:
        # rows that pair two windows: the double attends each window on its own
        import ctypes
        import importlib
        bg = importlib.import_module("dreamx-creator_b200.blockgrid")
        n_rows = params.shape[0]
        raw = (ctypes.c_int32 * (n_rows * bg.SPLIT_FIELDS)).from_address(int(geom.col_split))
        split = torch.tensor(list(raw), dtype=torch.int32).view(n_rows, bg.SPLIT_FIELDS)
        params = bg.unpair_rows(params, split, p_stride)
    params = params.numpy()
    if p_stride == 17:
        f_kv = int((params[:, 4] + params[:, 5]).max())
    else:
        f_kv = int((params[:, 6] + params[:, 7]).max())
    slots = [(geom.kv_slot0 + t) % geom.kv_slots for t in range(f_kv)]
    kf = torch.cat([k_hr[s * L:(s + 1) * L] for s in slots])
    vf = torch.cat([v_hr[s * L:(s + 1) * L] for s in slots])
    hr_base = 0
    if k_anchor is not None and anchor_mode:
        hr_base = k_anchor.shape[0]
        kf = torch.cat([k_anchor, kf])
        vf = torch.cat([v_anchor, vf])
    plan = {"params": params, "hr_base": hr_base, "p_stride": p_stride}
    o = owa.run_plan(q.reshape(q.shape[0], n, 128), kf.reshape(kf.shape[0], n, 128),
                     vf.reshape(vf.shape[0], n, 128), plan, f_cur=f, h=h, w=w,
                     kv_w=geom.kv_w)
    out.copy_(o.reshape(out.shape).to(BF16))
    return out
