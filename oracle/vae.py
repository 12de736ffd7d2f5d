"""Oracle: the Wan2.2 VAE decode on the CPU (test infrastructure only).

Restates ``WanVAE_.decode`` (video_refiner/wan/modules/vae2_2.py:812-844) for a
bf16 model: the latent un-normalisation, the 1x1x1 ``conv2``, then
``Decoder3d.forward`` (:672-724) one latent frame at a time over per-conv
feature caches, then ``unpatchify`` (:299-313). Each op is computed in
float64 over bf16 values and rounded to bf16 where the reference's bf16
tensor op rounds: conv outputs (bias included), F.normalize's norm and
quotient, the sqrt(C) and gamma products (RMS_norm :57-59), SiLU, the
residual adds. The caches follow the reference: a conv's cache is the last
two frames of its input, extended by the previous cache's last frame when
the call had one frame (:218-234); a CausalConv3d pads its front with zeros
for the frames the cache lacks (:34-42); upsample3d's time_conv skips its
first call ("Rep") and starts its cache from zeros (:112-148).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

CACHE_T = 2


def rb(x):
    """x rounded to bf16 (through fp32), kept in float64."""
    return x.to(torch.float32).to(torch.bfloat16).to(torch.float64)


def exact(x):
    """No rounding: the float64 restatement of the fp32 model."""
    return x


def causal_conv(x, w, b, cache, r=rb):
    """CausalConv3d (:17-42): x [C, T, H, W]; the cache's frames, then zeros for
    the rest of the 2 * pad_t front frames; spatial zero padding."""
    kt, kh = w.shape[2], w.shape[3]
    pt, ph = (kt - 1), kh // 2
    if cache is not None and pt > 0:
        x = torch.cat([cache, x], 1)
        pt -= cache.shape[1]
    x = F.pad(x, (ph, ph, ph, ph, pt, 0))
    y = F.conv3d(x[None], w.to(torch.float64), b.to(torch.float64))[0]
    return r(y)


def rms_norm(x, gamma, r=rb):
    """RMS_norm over the channels (dim 0 of [C, ...]) in bf16 steps."""
    C = x.shape[0]
    n = r(torch.sqrt((x * x).sum(0, keepdim=True)))
    n = torch.clamp_min(n, 1e-12 if r is exact else float(torch.tensor(1e-12).to(torch.bfloat16)))
    y = r(x / n)
    y = r(y * float(torch.tensor(math.sqrt(C), dtype=torch.float32)))
    return r(y * gamma.to(torch.float64).reshape(C, *([1] * (x.dim() - 1))))


def silu(x, r=rb):
    return r(x / (1 + torch.exp(-x)))


class Decoder:
    """Decoder3d with its caches (feat_cache / feat_idx as a list)."""

    def __init__(self, sd, *, dim_mult=(1, 2, 4, 4), num_res_blocks=2,
                 temperal_upsample=(True, True, False), bf16=True):
        """``bf16=False``: no rounding anywhere (the fp32 model, in float64)."""
        self.sd = {k: v.to(torch.float64) for k, v in sd.items()}
        self.r = rb if bf16 else exact
        self.dim_mult = list(dim_mult)
        self.nrb = num_res_blocks
        self.tup = list(temperal_upsample)

    # -- cached conv (:218-234, :686-697)
    def _cconv(self, x, pre):
        idx = self.idx[0]
        cache_x = x[:, -CACHE_T:].clone()
        old = self.cache[idx]
        if cache_x.shape[1] < 2 and old is not None and not isinstance(old, str):
            cache_x = torch.cat([old[:, -1:], cache_x], 1)
        y = causal_conv(x, self.sd[pre + ".weight"], self.sd[pre + ".bias"],
                        None if isinstance(old, str) else old, r=self.r)
        self.cache[idx] = cache_x
        self.idx[0] += 1
        return y

    def _res(self, x, pre):
        sd = self.sd
        if pre + ".shortcut.weight" in sd:
            h = causal_conv(x, sd[pre + ".shortcut.weight"], sd[pre + ".shortcut.bias"], None,
                            r=self.r)
        else:
            h = x
        y = silu(rms_norm(x, sd[pre + ".residual.0.gamma"], self.r), self.r)
        y = self._cconv(y, pre + ".residual.2")
        y = silu(rms_norm(y, sd[pre + ".residual.3.gamma"], self.r), self.r)
        y = self._cconv(y, pre + ".residual.6")
        return self.r(y + h)

    def _attn(self, x, pre):
        sd = self.sd
        C, T, H, W = x.shape
        n = rms_norm(x, sd[pre + ".norm.gamma"], self.r)
        qkv = self.r(torch.einsum("ct..., oc -> ot...", n,
                              sd[pre + ".to_qkv.weight"][:, :, 0, 0])
                 + sd[pre + ".to_qkv.bias"][:, None, None, None])
        qkv = qkv.reshape(3 * C, T, H * W).permute(1, 2, 0)        # [T, HW, 3C]
        q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]
        p = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(C), -1)
        o = self.r(p @ v)                                               # [T, HW, C]
        o = o.permute(2, 0, 1).reshape(C, T, H, W)
        y = self.r(torch.einsum("ct..., oc -> ot...", o, sd[pre + ".proj.weight"][:, :, 0, 0])
               + sd[pre + ".proj.bias"][:, None, None, None])
        return self.r(y + x)

    def _resample(self, x, pre, mode):
        sd = self.sd
        C, T, H, W = x.shape
        if mode == "upsample3d":
            idx = self.idx[0]
            old = self.cache[idx]
            if old is None:
                self.cache[idx] = "Rep"
                self.idx[0] += 1
            else:
                cache_x = x[:, -CACHE_T:].clone()
                rep_marker = isinstance(old, str)
                if cache_x.shape[1] < 2:
                    prev = torch.zeros_like(cache_x) if rep_marker else old[:, -1:]
                    cache_x = torch.cat([prev, cache_x], 1)
                y = causal_conv(x, sd[pre + ".time_conv.weight"], sd[pre + ".time_conv.bias"],
                                None if rep_marker else old, r=self.r)
                self.cache[idx] = cache_x
                self.idx[0] += 1
                y = y.reshape(2, C, T, H, W)
                x = torch.stack([y[0], y[1]], 2).reshape(C, 2 * T, H, W)
        T = x.shape[1]
        up = x.repeat_interleave(2, 2).repeat_interleave(2, 3)      # nearest(-exact) 2x
        y = F.conv2d(up.permute(1, 0, 2, 3), sd[pre + ".resample.1.weight"],
                     sd[pre + ".resample.1.bias"], padding=1)
        return self.r(y).permute(1, 0, 2, 3)

    @staticmethod
    def _dup_up(x, cout, ft, fs, first_chunk):
        """DupUp3D (:370-413)."""
        C, T, H, W = x.shape
        Fk = ft * fs * fs
        reps = cout * Fk // C
        y = x.repeat_interleave(reps, 0).reshape(cout, ft, fs, fs, T, H, W)
        y = y.permute(0, 4, 1, 5, 2, 6, 3).reshape(cout, T * ft, H * fs, W * fs)
        return y[:, ft - 1:] if first_chunk else y

    def _up_block(self, x, i, in_dim, out_dim, first_chunk):
        pre = f"decoder.upsamples.{i}"
        t_up = self.tup[i] if i < len(self.tup) else False
        up = i != len(self.dim_mult) - 1
        y = x
        for j in range(self.nrb + 1):
            y = self._res(y, f"{pre}.upsamples.{j}")
        if not up:
            return y
        y = self._resample(y, f"{pre}.upsamples.{self.nrb + 1}",
                           "upsample3d" if t_up else "upsample2d")
        s = self._dup_up(x, out_dim, 2 if t_up else 1, 2, first_chunk)
        return self.r(y + s)

    def frame(self, x, first_chunk):
        """Decoder3d.forward of x [z_dim, T, h, w] with the caches."""
        sd = self.sd
        self.idx = [0]
        x = self._cconv(x, "decoder.conv1")
        x = self._res(x, "decoder.middle.0")
        x = self._attn(x, "decoder.middle.1")
        x = self._res(x, "decoder.middle.2")
        dim = sd["decoder.conv1.weight"].shape[0] // self.dim_mult[-1]
        dims = [dim * u for u in [self.dim_mult[-1]] + self.dim_mult[::-1]]
        for i, (di, do) in enumerate(zip(dims[:-1], dims[1:])):
            x = self._up_block(x, i, di, do, first_chunk)
        x = silu(rms_norm(x, sd["decoder.head.0.gamma"], self.r), self.r)
        return self._cconv(x, "decoder.head.2")

    def decode(self, z, mean, std):
        """z [z_dim, T, h, w] (bf16 values), mean / std [z_dim] fp32 -> the raw
        decoded video [3, F, 16 h, 16 w] (float64 of bf16 values), unclamped."""
        sd = self.sd
        self.cache = [None] * 64
        C = z.shape[0]
        s1 = self.r(1.0 / self.r(std.to(torch.float64)))
        x = self.r(self.r(z.to(torch.float64) / s1[:, None, None, None]) + self.r(mean.to(torch.float64))
               [:, None, None, None])
        x = causal_conv(x, sd["conv2.weight"], sd["conv2.bias"], None, r=self.r)
        outs = [self.frame(x[:, i:i + 1], i == 0) for i in range(x.shape[1])]
        y = torch.cat(outs, 1)                                       # [12, F, H, W]
        c12, Fr, H, W = y.shape
        # unpatchify "b (c r q) f h w -> b c f (h q) (w r)"
        y = y.reshape(3, 2, 2, Fr, H, W).permute(0, 3, 4, 2, 5, 1).reshape(3, Fr, 2 * H, 2 * W)
        return y
