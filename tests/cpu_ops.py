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


# --------------------------------------------------------------------------- VAE decode
def emulate_conv3d(x, w2, bias, *, kt, kh, shuffle_t=1, up2_phase=-1, residual=None):
    """srdit_conv3d in float64: output frame o, pixel (h, w) sums, over taps (dt,
    ky, kx) and channels, x[o + dt, h + dy, w + dx] * w2[n, ((dt kh + ky) kh + kx)
    cin + c] with (dy, dx) = (ky - kh/2, kx - kh/2), or, for an up2 phase (i, j),
    (floor((i + ky - 1) / 2), floor((j + kx - 1) / 2)); zeros outside the frame;
    bf16 rounding; interleaved or phase stores as the kernel's."""
    Fi, H, W, cin = x.shape
    Fo = Fi - kt + 1
    cout = w2.shape[0]
    xp = torch.nn.functional.pad(x.double(), (0, 0, 1, 1, 1, 1))   # one zero pixel around
    pi, pj = (up2_phase >> 1, up2_phase & 1) if up2_phase >= 0 else (0, 0)
    cols = []
    for dt in range(kt):
        for ky in range(kh):
            for kx in range(kh):
                if up2_phase >= 0:
                    dy, dx = (pi + ky - 1) // 2, (pj + kx - 1) // 2
                else:
                    dy, dx = ky - kh // 2, kx - kh // 2
                cols.append(xp[dt:dt + Fo, 1 + dy:1 + dy + H, 1 + dx:1 + dx + W, :])
    a = torch.cat(cols, -1)
    y = (a @ w2.double().t() + bias.double()).to(torch.float32).to(torch.bfloat16).double()
    if up2_phase >= 0:
        out = torch.zeros(Fo, 2 * H, 2 * W, cout, dtype=torch.float64)
        out[:, pi::2, pj::2] = y
        y = out
    if residual is not None:
        y = (residual.double() + y).to(torch.float32).to(torch.bfloat16).double()
        if up2_phase >= 0:
            keep = torch.zeros(2 * H, 2 * W, dtype=torch.bool)
            keep[pi::2, pj::2] = True
            y = torch.where(keep[None, :, :, None], y, torch.zeros_like(y))
    if shuffle_t > 1:
        cg = cout // shuffle_t
        y = y.reshape(Fo, H, W, shuffle_t, cg).permute(0, 3, 1, 2, 4).reshape(Fo * shuffle_t,
                                                                                H, W, cg)
    return y


def conv3d(x, weight, bias, *, kt=1, kh=3, residual=None, res_scale=1.0, relu=False,
           shuffle=1, shuffle_t=1, up2_phase=-1, dup=None, out=None, status=None):
    """srdit_conv3d by its emulation (float64 sums, the kernel's bf16 roundings and
    stores); the DupUp3D gather of a phase launch as the materialised shortcut."""
    if res_scale != 1.0 or relu or shuffle != 1:
        raise NotImplementedError("the VAE decode's forms only")
    if dup is not None:
        import importlib
        vae = importlib.import_module("dreamx-creator_b200.vae")
        xd, ft, shift = dup
        residual = vae._dup_up(xd, weight.shape[0], ft, 2, shift > 0)
    y = emulate_conv3d(x, weight, bias, kt=kt, kh=kh, shuffle_t=shuffle_t, up2_phase=up2_phase,
                       residual=residual).to(torch.bfloat16)
    if up2_phase >= 0:
        pi, pj = up2_phase >> 1, up2_phase & 1
        out[:, pi::2, pj::2] = y[:, pi::2, pj::2]
        return out
    if out is not None:
        out.copy_(y)
        return out
    return y


def conv3d_weight(w, *, cin_pad=None):
    import importlib
    return importlib.import_module("dreamx-creator_b200.ops").conv3d_weight(w, cin_pad=cin_pad)


def rms_silu(x, gamma, *, silu=True, out=None):
    """srdit_rms_silu by the oracle's RMS_norm (+ SiLU) over the last dim."""
    from oracle import vae as ov
    y = ov.rms_norm(x.double().movedim(-1, 0), gamma.double())
    if silu:
        y = ov.silu(y)
    y = y.movedim(0, -1).to(torch.bfloat16)
    if out is None:
        return y
    out.copy_(y)
    return out


def vae_attend(q, k, v):
    """The middle block's attention as the oracle computes it (float64 softmax,
    the output rounded to bf16)."""
    import math
    qd, kd, vd = q.double(), k.double(), v.double()
    p = torch.softmax(qd @ kd.transpose(-1, -2) / math.sqrt(q.shape[-1]), -1)
    return (p @ vd).to(torch.float32).to(torch.bfloat16)

