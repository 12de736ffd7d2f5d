"""Wan2.2 VAE decode on the B200 kernels (``srdit_conv3d``, ``srdit_rms_silu``).

The reference decodes the refined latent with ``WanVAE_.decode``
(video_refiner/wan/modules/vae2_2.py:812-844: un-normalise, the 1x1x1
``conv2``, then ``Decoder3d`` one latent frame at a time over per-conv feature
caches, then ``unpatchify``; the pipeline's wrapper, utils/sr_dit_wrapper.py:
27-100, runs it in bf16 and clamps to [-1, 1]). This module keeps that
structure and its cache semantics, on channels-last frames [T, H, W, C]:

  * every CausalConv3d is one ``srdit_conv3d`` launch over a *causal history*
    buffer [2 + T, H, W, C]: the conv's previous input frames (zeros before
    the first call -- the causal padding) followed by this call's frames; after
    the call its last two frames move to the front, which is the reference's
    ``feat_cache`` update (:218-234) including its "fewer than two new frames"
    case;
  * RMS_norm + SiLU (``srdit_rms_silu``) writes straight into the history of
    the conv that follows it; the residual adds (ResidualBlock :236, the
    Up_ResidualBlock shortcut :495) run in the epilogue of the conv that ends
    the branch;
  * Resample "upsample3d" (:112-148): the time_conv (3x1x1, C -> 2C) stores its
    two channel halves as interleaved frames (``shuffle_t``), skipping its
    first call as the reference's "Rep" marker does; nearest 2x + Conv2d is
    four phase launches of the conv on the low-resolution frame (``up2_phase``);
  * AttentionBlock (:238-278): RMS_norm, the 1x1 qkv / proj convs on the conv
    kernel, single-head attention over a frame's pixels by torch's
    scaled_dot_product_attention (a library kernel, as in the reference);
  * DupUp3D (:370-413) is gathered from the block input by the resample's
    phase launches (``srdit_dup_up``) and added there;
  * unpatchify (:299-313) and the latent un-normalisation are index plumbing
    in torch.

Channel counts must be multiples of 64 except the latent (48, zero-padded) and
the 12 output channels.
"""
from __future__ import annotations

import torch

from . import _lib
from . import ops as _ops

# The kernel launchers the decoder calls (the libsrdit_b200.so wrappers). A test
# may point this at a table of its own to run the host-side orchestration
# without a GPU; the module has no other compute path.
ops = _ops
# single-head attention of the middle block (a library kernel, as in the reference)
attend = torch.nn.functional.scaled_dot_product_attention


def _pad64(c):
    return (c + 63) // 64 * 64


class _Conv:
    """A CausalConv3d / Conv2d in srdit_conv3d's layout (weights K-major, fp32
    bias), with the causal history buffer of a kt = 3 conv."""

    def __init__(self, sd, prefix, device, cout_pad=None):
        w, b = sd[prefix + ".weight"], sd[prefix + ".bias"]
        if w.dim() == 4:
            w = w[:, :, None]
        self.cout, self.cin, self.kt, self.kh = w.shape[0], w.shape[1], w.shape[2], w.shape[3]
        self.cin_pad = _pad64(self.cin)
        self.cout_pad = cout_pad or self.cout
        wp = w
        if self.cout_pad != self.cout:
            wp = torch.nn.functional.pad(w.float(), (0, 0, 0, 0, 0, 0, 0, 0, 0,
                                                     self.cout_pad - self.cout))
            b = torch.nn.functional.pad(b.float(), (0, self.cout_pad - self.cout))
        self.w = ops.conv3d_weight(wp, cin_pad=self.cin_pad).to(device)
        self.b = b.detach().to(device, torch.float32).contiguous()
        self.hist = None      # [2 + T, H, W, cin_pad]: history frames, then this call's
        self.calls = 0

    def history(self, T, H, W, device):
        """The history buffer for a call of T frames (its frames [2, 2 + T) are
        this call's input, to be filled by the caller)."""
        shape = (2 + T, H, W, self.cin_pad)
        h = self.hist
        if h is None or h.shape[1:] != shape[1:] or h.shape[0] < shape[0]:
            big = torch.zeros((max(2 + T, 6),) + shape[1:], dtype=torch.bfloat16, device=device)
            if h is not None and h.shape[1:] == shape[1:]:
                big[:2] = h[:2]
            self.hist = h = big
        return h[:2 + T]

    def run_history(self, hist, T, **kw):
        """The conv over hist [2 + T, ...] (kt = 3), then the cache update."""
        y = ops.conv3d(hist, self.w, self.b, kt=3, kh=self.kh, **kw)
        # frames T, T + 1 to the front, in order (they overlap frames 0, 1 when T = 1)
        hist[0].copy_(hist[T])
        hist[1].copy_(hist[T + 1])
        self.calls += 1
        return y

    def __call__(self, x, **kw):
        """kt = 1: the conv of x [T, H, W, cin_pad] itself."""
        return ops.conv3d(x, self.w, self.b, kt=1, kh=self.kh, **kw)


def _pad_channels(x, c):
    return x if x.shape[-1] == c else torch.nn.functional.pad(x, (0, c - x.shape[-1]))


class _ResBlock:
    """ResidualBlock (vae2_2.py:193-236): shortcut(x) + conv2(silu(norm2(conv1(
    silu(norm1(x)))))) with both convs causal over their caches."""

    def __init__(self, sd, prefix, device):
        self.g1 = sd[prefix + ".residual.0.gamma"].reshape(-1).to(device, torch.bfloat16)
        self.c1 = _Conv(sd, prefix + ".residual.2", device)
        self.g2 = sd[prefix + ".residual.3.gamma"].reshape(-1).to(device, torch.bfloat16)
        self.c2 = _Conv(sd, prefix + ".residual.6", device)
        self.short = _Conv(sd, prefix + ".shortcut", device) if prefix + ".shortcut.weight" in sd \
            else None

    def __call__(self, x, residual=None):
        T, H, W, _ = x.shape
        dev = x.device
        h = self.short(x) if self.short is not None else x
        h1 = self.c1.history(T, H, W, dev)
        ops.rms_silu(x, self.g1, out=h1[2:])
        y = self.c1.run_history(h1, T)
        h2 = self.c2.history(T, H, W, dev)
        ops.rms_silu(y, self.g2, out=h2[2:])
        return self.c2.run_history(h2, T, residual=h)


class _Attention:
    """AttentionBlock (vae2_2.py:238-278): x + proj(attn(qkv(norm(x)))) per frame."""

    def __init__(self, sd, prefix, device):
        self.g = sd[prefix + ".norm.gamma"].reshape(-1).to(device, torch.bfloat16)
        self.qkv = _Conv(sd, prefix + ".to_qkv", device)
        self.proj = _Conv(sd, prefix + ".proj", device)

    def __call__(self, x):
        T, H, W, C = x.shape
        n = ops.rms_silu(x, self.g, silu=False)
        qkv = self.qkv(n).view(T, 1, H * W, 3 * C)
        q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
        o = attend(q, k, v)
        return self.proj(o.reshape(T, H, W, C).contiguous(), residual=x)


class _Resample:
    """Resample "upsample2d" / "upsample3d" (vae2_2.py:71-148) up to the final
    2x nearest + Conv2d, whose launches add the block's DupUp3D shortcut."""

    def __init__(self, sd, prefix, mode, device):
        self.mode = mode
        self.conv = _Conv(sd, prefix + ".resample.1", device)
        self.time = _Conv(sd, prefix + ".time_conv", device) if mode == "upsample3d" else None

    def __call__(self, x, dup):
        T, H, W, C = x.shape
        if self.time is not None:
            if self.time.calls == 0:
                # the first call only marks the cache ("Rep"): no time_conv,
                # and the history keeps its zeros
                self.time.calls = 1
            else:
                h = self.time.history(T, H, W, x.device)
                h[2:].copy_(x)
                x = self.time.run_history(h, T, shuffle_t=2)
                T = x.shape[0]
        out = torch.empty(T, 2 * H, 2 * W, self.conv.cout, dtype=torch.bfloat16, device=x.device)
        for ph in range(4):
            self.conv(x, up2_phase=ph, out=out, dup=dup)
        return out


def _dup_up(x, cout, ft, fs, first_chunk):
    """DupUp3D (vae2_2.py:370-413) on channels-last frames: output channel c of
    frame t * ft + a, pixel (h fs + i, w fs + j) is input channel (c F + a fs^2 +
    i fs + j) // repeats of frame t, pixel (h, w), F = ft fs^2; a clip's first
    call drops the first ft - 1 frames."""
    T, H, W, cin = x.shape
    F = ft * fs * fs
    repeats = cout * F // cin
    c = torch.arange(cout, device=x.device)
    idx = (c[None, None, None, :] * F
           + torch.arange(ft, device=x.device)[:, None, None, None] * fs * fs
           + torch.arange(fs, device=x.device)[None, :, None, None] * fs
           + torch.arange(fs, device=x.device)[None, None, :, None]) // repeats
    g = x[..., idx.reshape(-1)].reshape(T, H, W, ft, fs, fs, cout)
    y = g.permute(0, 3, 1, 4, 2, 5, 6).reshape(T * ft, H * fs, W * fs, cout)
    if first_chunk:
        y = y[ft - 1:]
    return y.contiguous()


class _UpBlock:
    """Up_ResidualBlock (vae2_2.py:455-497)."""

    def __init__(self, sd, prefix, in_dim, out_dim, mult, t_up, up, device):
        self.res = [_ResBlock(sd, f"{prefix}.upsamples.{j}", device) for j in range(mult)]
        self.resample = (_Resample(sd, f"{prefix}.upsamples.{mult}",
                                   "upsample3d" if t_up else "upsample2d", device)
                         if up else None)
        self.dup = (out_dim, 2 if t_up else 1, 2) if up else None

    def __call__(self, x, first_chunk):
        y = x
        for rb in self.res:
            y = rb(y)
        if self.resample is None:
            return y
        _, ft, _ = self.dup
        # the DupUp3D shortcut of x, added by the resample's phase launches
        return self.resample(y, dup=(x, ft, ft - 1 if first_chunk else 0))


class Wan22VAEDecoder:
    """``WanVAE_.decode`` + the wrapper's clamp for the Wan2.2 VAE (z_dim 48,
    dec_dim 256, dim_mult [1, 2, 4, 4], 2 residual blocks, temporal upsampling
    [True, True, False]); weights from the reference ``WanVAE_`` state dict
    (its ``conv2.*`` and ``decoder.*`` entries). Call ``decode(z, mean, std)``
    on a latent [48, T, h, w]; returns the video [3, 1 + 4 (T - 1), 16 h, 16 w]
    fp32 in [-1, 1]."""

    def __init__(self, sd, *, dim=256, z_dim=48, dim_mult=(1, 2, 4, 4), num_res_blocks=2,
                 temperal_upsample=(True, True, False), device="cuda"):
        self.device = torch.device(device)
        dev = self.device
        dims = [dim * u for u in [dim_mult[-1]] + list(dim_mult[::-1])]
        if any(d % 64 for d in dims):
            raise _lib.SrditError(f"decoder widths {dims}: multiples of 64 are needed")
        self.z_dim = z_dim
        self.conv2 = _Conv(sd, "conv2", dev)
        self.conv1 = _Conv(sd, "decoder.conv1", dev)
        self.middle = [_ResBlock(sd, "decoder.middle.0", dev),
                       _Attention(sd, "decoder.middle.1", dev),
                       _ResBlock(sd, "decoder.middle.2", dev)]
        self.ups = []
        for i, (di, do) in enumerate(zip(dims[:-1], dims[1:])):
            t_up = temperal_upsample[i] if i < len(temperal_upsample) else False
            self.ups.append(_UpBlock(sd, f"decoder.upsamples.{i}", di, do, num_res_blocks + 1,
                                     t_up, i != len(dim_mult) - 1, dev))
        self.head_g = sd["decoder.head.0.gamma"].reshape(-1).to(dev, torch.bfloat16)
        self.head = _Conv(sd, "decoder.head.2", dev, cout_pad=16)

    @staticmethod
    def param_shapes(dim=256, z_dim=48, dim_mult=(1, 2, 4, 4), num_res_blocks=2,
                     temperal_upsample=(True, True, False)):
        """{name: shape} of the decoder parameters of the reference ``WanVAE_``
        state dict (``conv2.*``, ``decoder.*``)."""
        dims = [dim * u for u in [dim_mult[-1]] + list(dim_mult[::-1])]
        shp = {"conv2.weight": (z_dim, z_dim, 1, 1, 1), "conv2.bias": (z_dim,),
               "decoder.conv1.weight": (dims[0], z_dim, 3, 3, 3), "decoder.conv1.bias": (dims[0],)}

        def res(pre, i, o):
            shp[pre + ".residual.0.gamma"] = (i, 1, 1, 1)
            shp[pre + ".residual.2.weight"] = (o, i, 3, 3, 3)
            shp[pre + ".residual.2.bias"] = (o,)
            shp[pre + ".residual.3.gamma"] = (o, 1, 1, 1)
            shp[pre + ".residual.6.weight"] = (o, o, 3, 3, 3)
            shp[pre + ".residual.6.bias"] = (o,)
            if i != o:
                shp[pre + ".shortcut.weight"] = (o, i, 1, 1, 1)
                shp[pre + ".shortcut.bias"] = (o,)

        d0 = dims[0]
        res("decoder.middle.0", d0, d0)
        shp["decoder.middle.1.norm.gamma"] = (d0, 1, 1)
        shp["decoder.middle.1.to_qkv.weight"] = (3 * d0, d0, 1, 1)
        shp["decoder.middle.1.to_qkv.bias"] = (3 * d0,)
        shp["decoder.middle.1.proj.weight"] = (d0, d0, 1, 1)
        shp["decoder.middle.1.proj.bias"] = (d0,)
        res("decoder.middle.2", d0, d0)
        for i, (di, do) in enumerate(zip(dims[:-1], dims[1:])):
            pre = f"decoder.upsamples.{i}.upsamples"
            c = di
            for j in range(num_res_blocks + 1):
                res(f"{pre}.{j}", c, do)
                c = do
            if i != len(dim_mult) - 1:
                r = f"{pre}.{num_res_blocks + 1}"
                shp[r + ".resample.1.weight"] = (do, do, 3, 3)
                shp[r + ".resample.1.bias"] = (do,)
                if i < len(temperal_upsample) and temperal_upsample[i]:
                    shp[r + ".time_conv.weight"] = (2 * do, do, 3, 1, 1)
                    shp[r + ".time_conv.bias"] = (2 * do,)
        shp["decoder.head.0.gamma"] = (dims[-1], 1, 1, 1)
        shp["decoder.head.2.weight"] = (12, dims[-1], 3, 3, 3)
        shp["decoder.head.2.bias"] = (12,)
        return shp

    @classmethod
    def seeded_state_dict(cls, seed=0, **kw):
        """Seeded random bf16 weights with the reference's names and shapes (runs
        without a checkpoint): gammas 1 + 0.2 N(0, 1), conv weights N(0, 1) /
        sqrt(fan_in), biases 0.05 N(0, 1)."""
        g = torch.Generator().manual_seed(seed)
        sd = {}
        for n, shape in cls.param_shapes(**kw).items():
            t = torch.randn(*shape, generator=g)
            if n.endswith(".gamma"):
                t = 1 + 0.2 * t
            elif n.endswith(".bias"):
                t = 0.05 * t
            else:
                fan = 1
                for d in shape[1:]:
                    fan *= d
                t = t / fan ** 0.5
            sd[n] = t.to(torch.bfloat16)
        return sd

    def flops(self, T, h, w):
        """Algorithmic conv + attention FLOPs of ``decode`` on a [z, T, h, w]
        latent (2 per multiply-add; the first frame decodes to 1 frame, later
        ones to 4 through the temporal upsampling)."""
        tot = 2 * T * h * w * self.conv2.cout * self.conv2.cin
        for i in range(T):
            tot += self._frame_flops(h, w, first=(i == 0))
        return tot

    def _frame_flops(self, h, w, first):
        def conv(c, t, hh, ww):
            return 2 * t * hh * ww * c.cout * c.cin * c.kt * c.kh * c.kh
        t, hh, ww = 1, h, w
        f = conv(self.conv1, t, hh, ww)
        for blk in self.middle:
            if isinstance(blk, _ResBlock):
                f += conv(blk.c1, t, hh, ww) + conv(blk.c2, t, hh, ww)
            else:
                C = blk.qkv.cin
                f += conv(blk.qkv, t, hh, ww) + conv(blk.proj, t, hh, ww)
                f += 4 * t * (hh * ww) ** 2 * C
        for ub in self.ups:
            for rb in ub.res:
                f += conv(rb.c1, t, hh, ww) + conv(rb.c2, t, hh, ww)
                if rb.short is not None:
                    f += conv(rb.short, t, hh, ww)
            if ub.resample is not None:
                if ub.resample.time is not None and not first:
                    f += conv(ub.resample.time, t, hh, ww)
                    t *= 2
                f += 4 * conv(ub.resample.conv, t, hh, ww)
                hh, ww = 2 * hh, 2 * ww
        c = self.head
        f += 2 * t * hh * ww * c.cout * c.cin * 27
        return f

    def _convs(self):
        out = [self.conv1, self.head]
        for blk in self.middle:
            if isinstance(blk, _ResBlock):
                out += [blk.c1, blk.c2]
        for ub in self.ups:
            for rb in ub.res:
                out += [rb.c1, rb.c2]
            if ub.resample is not None and ub.resample.time is not None:
                out.append(ub.resample.time)
        return out

    def clear_cache(self):
        """A new clip: every conv's history back to zeros (vae2_2.py:858-866)."""
        for c in self._convs():
            c.hist = None
            c.calls = 0

    def _decoder(self, x, first_chunk):
        """Decoder3d.forward (vae2_2.py:672-724) of one latent frame x [1, h, w, 64]."""
        T, H, W, _ = x.shape
        h = self.conv1.history(T, H, W, x.device)
        h[2:].copy_(x)
        x = self.conv1.run_history(h, T)
        x = self.middle[0](x)
        x = self.middle[1](x)
        x = self.middle[2](x)
        for ub in self.ups:
            x = ub(x, first_chunk)
        T, H, W, _ = x.shape
        hh = self.head.history(T, H, W, x.device)
        ops.rms_silu(x, self.head_g, out=hh[2:])
        return self.head.run_history(hh, T)[..., :self.head.cout]

    def decode(self, z, mean, std, clamp=True):
        """z [z_dim, T, h, w] (any float dtype) -> video [3, F, 16 h, 16 w] fp32,
        clamped to [-1, 1] as the pipeline's wrapper does (``clamp=False``: the
        raw ``WanVAE_.decode`` output)."""
        dev = self.device
        self.clear_cache()
        C, T, h, w = z.shape
        if C != self.z_dim:
            raise ValueError(f"latent of {C} channels, expected {self.z_dim}")
        zb = z.to(dev, torch.bfloat16).permute(1, 2, 3, 0)          # [T, h, w, C]
        # z / scale[1] + scale[0] with scale = [mean, 1 / std] in the model dtype
        s1 = (1.0 / std.to(dev, torch.bfloat16)).to(torch.bfloat16)
        zb = zb / s1 + mean.to(dev, torch.bfloat16)
        x = self.conv2(_pad_channels(zb.contiguous(), self.conv2.cin_pad))
        x = _pad_channels(x, self.conv1.cin_pad)
        frames = []
        for i in range(T):
            frames.append(self._decoder(x[i:i + 1].contiguous(), first_chunk=(i == 0)))
        out = torch.cat(frames)                                       # [F, 8h, 8w, 12]
        F_, H, W, _ = out.shape
        # unpatchify, "b (c r q) f h w -> b c f (h q) (w r)" with q = r = 2
        v = out.view(F_, H, W, 3, 2, 2).permute(3, 0, 1, 5, 2, 4).reshape(3, F_, 2 * H, 2 * W)
        self.clear_cache()
        v = v.float()
        return v.clamp_(-1, 1) if clamp else v
