"""Drop-in ``Fp8Linear`` on the B200 e4m3 GEMM.

Interface of the reference module (video_refiner/wan/modules/sr_dit/fp8_linear.py:
214-354): ``Fp8Linear(weight, bias)`` / ``Fp8Linear.from_linear(lin)``, the
buffers ``weight_fp8`` (e4m3 [N, K]), ``weight_scale`` (fp32 [1, N]), ``bias``
(bf16 [N]) and the zero-element ``weight`` stand-in that keeps
``self.o.weight.dtype`` working (models.py:673, :1013), ``forward(x[..., K]) ->
[..., N]`` in x's dtype, ``TARGETS_ALL`` and ``convert_linears_to_fp8(model,
targets, skip_first, skip_last, blocks_attr)``.

The weight is quantised once, per output channel, with the reference's
row-wise rule (fp8_linear.py:93-103); every call quantises the activation per
token (``srdit_quant_rowwise``) and runs the row-wise scaled tcgen05 GEMM with
the bias in its epilogue (``srdit_fp8_gemm``). There is no torch._scaled_mm or
CPU path: without the library or a GPU, the call raises.
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

    # buffers whose dtype is part of their meaning: a module-wide dtype cast
    # (``.to(torch.bfloat16)``, ``.half()``, ``.float()``) must only move them
    _FIXED_DTYPE = {"weight_fp8": FP8_DTYPE, "weight_scale": torch.float32,
                    "bias": torch.bfloat16}

    def __init__(self, weight, bias=None):
        super().__init__()
        if weight.dim() != 2:
            raise ValueError(f"Fp8Linear needs a 2-D [out, in] weight, got {tuple(weight.shape)}")
        n_out, n_in = (int(v) for v in weight.shape)
        self.out_features, self.in_features = n_out, n_in
        q, s = quantize_weight(weight)
        self.register_buffer("weight_fp8", q.contiguous(), persistent=False)
        self.register_buffer("weight_scale", s.float().view(1, n_out).contiguous(),
                             persistent=False)
        # the GEMM epilogue adds a bf16 bias to the fp32 accumulator
        self.register_buffer("bias", None if bias is None else
                             bias.detach().to(torch.bfloat16).clone().contiguous(),
                             persistent=False)
        # zero-element stand-in: callers read .weight.dtype; any use as a real
        # weight fails on its shape instead of computing with stale values
        self.register_buffer("weight", weight.new_empty(0), persistent=False)

    @classmethod
    def from_linear(cls, lin: nn.Linear) -> "Fp8Linear":
        return cls(lin.weight, lin.bias).to(lin.weight.device)

    def _apply(self, fn, recurse=True):
        """Module-wide conversions move the fixed-dtype buffers, never cast them.

        The fixed buffers are hidden from ``fn`` while the base class converts
        the rest; ``fn`` is then applied to an empty probe tensor to learn the
        device it sends tensors to, and the original buffers are moved there
        unchanged (a bf16 round trip of the fp32 scales, or fp8 codes cast as
        numbers, would silently change the product)."""
        fixed = {}
        for name in self._FIXED_DTYPE:
            buf = self._buffers.get(name)
            if buf is not None:
                fixed[name] = buf
                self._buffers[name] = None
        try:
            super()._apply(fn, recurse)
        finally:
            if fixed:
                home = next(iter(fixed.values())).device
                dest = fn(torch.empty(0, device=home)).device
                for name, buf in fixed.items():
                    self._buffers[name] = buf if buf.device == dest else buf.to(dest)
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., in_features] -> [..., out_features] in x's dtype (computed from
        x rounded to bf16, the quantiser's input type)."""
        if x.shape[-1] != self.in_features:
            raise ValueError(f"Fp8Linear expects {self.in_features} input features, "
                             f"got {x.shape[-1]}")
        rows = x.reshape(-1, self.in_features)
        rows = rows.to(torch.bfloat16).contiguous()  # a view when x is contiguous bf16
        xq, xs = ops.quant_rowwise(rows)
        y = ops.fp8_gemm(xq, xs, self.weight_fp8, self.weight_scale.view(-1), self.bias)
        return y.to(x.dtype).view(*x.shape[:-1], self.out_features)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, fp8=e4m3-rowwise, backend=b200")


def convert_linears_to_fp8(model: nn.Module, targets=TARGETS_ALL, skip_first=0, skip_last=0,
                           blocks_attr="blocks"):
    """Replace the ``targets`` Linears of ``model.<blocks_attr>[i]`` by Fp8Linear,
    in place, for block indices skip_first <= i < len(blocks) - skip_last.

    Targets are dotted paths inside a block (``"self_attn.q"``, ``"ffn.0"``).
    A missing path, or one that is not an ``nn.Linear`` (for instance an
    Fp8Linear from an earlier call), is left alone, so the call is idempotent.
    Returns the qualified names converted, e.g. ``"blocks.3.ffn.0"``.
    """
    if not torch.cuda.is_available():
        raise _lib.SrditError("Fp8Linear needs a CUDA device (there is no CPU path)")
    blocks = getattr(model, blocks_attr, None)
    if blocks is None:
        return []
    chosen = range(int(skip_first), len(blocks) - int(skip_last))
    converted = []
    for idx in chosen:
        block = blocks[idx]
        for path in targets:
            try:
                lin = block.get_submodule(path)
            except AttributeError:
                continue
            if not isinstance(lin, nn.Linear):
                continue
            owner_path, _, leaf = path.rpartition(".")
            owner = block.get_submodule(owner_path) if owner_path else block
            owner.add_module(leaf, Fp8Linear.from_linear(lin))
            converted.append(f"{blocks_attr}.{idx}.{path}")
    return converted
