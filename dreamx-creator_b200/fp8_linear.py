"""Drop-in ``Fp8Linear`` on the B200 e4m3 GEMM.

Mirrors the reference module (video_refiner/wan/modules/sr_dit/fp8_linear.py:214-354):
the weight is quantised once, per output channel, to e4m3 with the reference's
row-wise rule; each call quantises the activation per token and runs the
row-wise scaled GEMM with the bias in the epilogue, returning bf16. The module
swap ``convert_linears_to_fp8`` and the ``weight`` stand-in that keeps
``self.o.weight.dtype`` working are the reference's interface.

The per-call path is two kernels of libsrdit_b200.so (row-wise quantiser +
tcgen05 GEMM); there is no torch._scaled_mm or CPU path.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib, ops

FP8_DTYPE = torch.float8_e4m3fn
FP8_MAX = 448.0

TARGETS_ALL = (
    "self_attn.q", "self_attn.k", "self_attn.v", "self_attn.o",
    "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.o",
    "ffn.0", "ffn.2",
)
TARGETS_FFN = ("ffn.0", "ffn.2")


def quantize_weight(weight: torch.Tensor):
    """Per-output-channel e4m3 of a [N, K] weight -> (e4m3 [N, K], fp32 scale [N]).

    One-time model preparation, the reference's row-wise rule
    (fp8_linear.py:93-103): scale = max(amax/448, 1e-12), q = e4m3(clamp(w/scale)).
    bf16 CUDA weights go through the library's quantiser; anything else is
    prepared with the same arithmetic in torch, once, at load time.
    """
    w = weight.detach()
    if w.is_cuda and w.dtype == torch.bfloat16 and w.shape[1] % 256 == 0:
        q, s = ops.quant_rowwise(w.contiguous())
        return q, s
    amax = w.abs().amax(dim=-1, keepdim=True).float()
    s = (amax / FP8_MAX).clamp_min(1e-12)
    q = (w.float() / s).clamp(-FP8_MAX, FP8_MAX).to(FP8_DTYPE)
    return q, s.reshape(-1).contiguous()


class Fp8Linear(nn.Module):
    """Frozen inference Linear computed as a row-wise scaled e4m3 GEMM."""

    def __init__(self, weight, bias=None):
        super().__init__()
        if weight.dim() != 2:
            raise ValueError(f"expected a 2D weight, got {tuple(weight.shape)}")
        self.out_features, self.in_features = weight.shape
        w_fp8, w_scale = quantize_weight(weight)
        self.register_buffer("weight_fp8", w_fp8.contiguous(), persistent=False)
        self.register_buffer("weight_scale", w_scale.reshape(1, -1).contiguous().float(),
                             persistent=False)
        if bias is None:
            self.bias = None
        else:
            b = bias.detach().clone()
            if b.dtype != torch.bfloat16:
                b = b.to(torch.bfloat16)
            self.register_buffer("bias", b.contiguous(), persistent=False)
        self.register_buffer("weight", torch.empty(0, dtype=weight.dtype, device=weight.device),
                             persistent=False)

    @classmethod
    def from_linear(cls, lin):
        return cls(lin.weight, lin.bias).to(lin.weight.device)

    def _apply(self, fn, recurse=True):
        saved = {n: b for n, b in self._buffers.items()
                 if n in ("weight_fp8", "weight_scale", "bias") and b is not None}
        out = super()._apply(fn, recurse)
        for name, old in saved.items():
            new = out._buffers[name]
            if new is not None and new.dtype != old.dtype:
                out._buffers[name] = old.to(device=new.device)
        return out

    def forward(self, x):
        out_dtype = x.dtype
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        xq, xs = ops.quant_rowwise(x2)
        out = ops.fp8_gemm(xq, xs, self.weight_fp8, self.weight_scale.reshape(-1), self.bias)
        if out_dtype is not torch.bfloat16:
            out = out.to(out_dtype)
        return out.reshape(*lead, self.out_features)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, fp8=e4m3-rowwise, backend=b200")


def convert_linears_to_fp8(model, targets=TARGETS_ALL, skip_first=0, skip_last=0,
                           blocks_attr="blocks"):
    """Swap the target Linears inside ``model.blocks`` for Fp8Linear, in place
    (fp8_linear.py:313-354). Returns the converted qualified names."""
    if not torch.cuda.is_available():
        raise _lib.SrditError("Fp8Linear needs a CUDA device (there is no CPU path)")
    blocks = getattr(model, blocks_attr, None)
    if blocks is None:
        return []
    n = len(blocks)
    lo, hi = int(skip_first), n - int(skip_last)
    converted = []
    for i, block in enumerate(blocks):
        if not (lo <= i < hi):
            continue
        for suffix in targets:
            *path, leaf = suffix.split(".")
            parent = block
            for p in path:
                parent = getattr(parent, p, None) if not p.isdigit() else parent[int(p)]
                if parent is None:
                    break
            if parent is None:
                continue
            cur = parent[int(leaf)] if leaf.isdigit() else getattr(parent, leaf, None)
            if not isinstance(cur, nn.Linear):
                continue
            new = Fp8Linear.from_linear(cur)
            if leaf.isdigit():
                parent[int(leaf)] = new
            else:
                setattr(parent, leaf, new)
            converted.append(f"{blocks_attr}.{i}.{suffix}")
    return converted
