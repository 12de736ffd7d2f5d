"""Oracle: fp8 quantisation, fp8 Linear, norms, RoPE (test infrastructure only).

Restates, with numpy / torch on the CPU:
  * ``_quantize_rowwise_impl`` -- video_refiner/wan/modules/sr_dit/fp8_linear.py:93-103
  * ``Fp8Linear.__init__/forward`` -- fp8_linear.py:223-297 (the row-wise scaled
    GEMM ``torch._scaled_mm(xq, w.t(), scale_a, scale_b, bias)``, restated as the
    algebraically identical dequantised product, since CPU ``_scaled_mm`` only
    takes per-tensor scales)
  * ``WanLayerNorm.forward`` (non-DTensor branch) -- models.py:497-503
  * ``WanRMSNorm.forward`` -- models.py:424-440
  * ``rope_params`` / ``_rope_axis_dims`` / ``rope_apply`` -- models.py:80-97, 173-214
  * the GELU(tanh) of ``ffn`` -- models.py:1200-1202
"""
from __future__ import annotations

import math

import numpy as np
import torch

FP8_MAX = 448.0


def quantize_rowwise(x: torch.Tensor):
    """fp8_linear.py:93-103: (e4m3 [..., K], fp32 scale [..., 1])."""
    amax = x.abs().amax(dim=-1, keepdim=True).float()
    scale = (amax / FP8_MAX).clamp_min(1e-12)
    q = (x.float() / scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, scale


def fp8_linear_weights(weight: torch.Tensor):
    """Fp8Linear.__init__ (fp8_linear.py:228-234): per-output-channel e4m3."""
    wq, ws = quantize_rowwise(weight.detach())
    return wq, ws.reshape(-1).float()


def fp8_linear(x: torch.Tensor, wq, ws, bias=None, acc_dtype=torch.float64):
    """Fp8Linear.forward (fp8_linear.py:282-297), bf16 out.

    The row-wise scaled product sum_k xq*wq * sa[m]*sb[n] + bias, accumulated in
    ``acc_dtype``, rounded once to bf16.
    """
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    xq, xs = quantize_rowwise(x2)
    acc = xq.to(acc_dtype) @ wq.to(acc_dtype).t()
    y = acc * xs.to(acc_dtype) * ws.reshape(1, -1).to(acc_dtype)
    if bias is not None:
        y = y + bias.to(acc_dtype)
    return y.to(torch.bfloat16).reshape(*lead, wq.shape[0])


def layer_norm(x: torch.Tensor, eps=1e-6, weight=None, bias=None):
    """WanLayerNorm.forward (models.py:497-503): fp32 layer_norm, back to x's dtype."""
    w = weight.float() if weight is not None else None
    b = bias.float() if bias is not None else None
    return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), w, b, eps).type_as(x)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps=1e-6):
    """WanRMSNorm.forward (models.py:437-440)."""
    xf = x.float()
    n = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return n.type_as(x) * weight


def gelu_tanh(x: torch.Tensor):
    """nn.GELU(approximate='tanh') (models.py:1201)."""
    return torch.nn.functional.gelu(x, approximate="tanh")


def rope_axis_dims(head_dim: int):
    """models.py:91-97."""
    return (head_dim - 4 * (head_dim // 6), 2 * (head_dim // 6), 2 * (head_dim // 6))


def rope_params(max_seq_len, dim, theta=10000.0):
    """models.py:80-88: complex128 [max_seq_len, dim/2]."""
    freqs = torch.outer(torch.arange(max_seq_len),
                        1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float64).div(dim)))
    return torch.polar(torch.ones_like(freqs), freqs)


def rope_freqs(max_seq_len=1024, head_dim=128, theta=10000.0):
    """WanModel._build_rope_freqs (models.py:1724-1737)."""
    t, h, w = rope_axis_dims(head_dim)
    return torch.cat([rope_params(max_seq_len, t, theta), rope_params(max_seq_len, h, theta),
                      rope_params(max_seq_len, w, theta)], dim=1)


def rope_apply(x: torch.Tensor, grid, freqs, t_offset=0):
    """rope_apply for one sample (models.py:173-214): x [f*h*w, n, d] -> same dtype."""
    f, h, w = grid
    n, c = x.shape[1], x.shape[2] // 2
    fs = freqs.split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    seq = f * h * w
    xc = torch.view_as_complex(x[:seq].to(torch.float64).reshape(seq, n, -1, 2))
    fr = torch.cat([fs[0][t_offset:t_offset + f].view(f, 1, 1, -1).expand(f, h, w, -1),
                    fs[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                    fs[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(seq, 1, -1)
    return torch.view_as_real(xc * fr).flatten(2).to(x.dtype)


def rope_tables(freqs: torch.Tensor):
    """(cos, sin) float64 [rows, 64] of the complex table."""
    return freqs.real.contiguous(), freqs.imag.contiguous()


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return float(torch.linalg.vector_norm(a - b) / max(float(torch.linalg.vector_norm(b)), 1e-30))


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().reshape(-1)
    b = b.double().reshape(-1)
    return float(torch.dot(a, b) / (torch.linalg.vector_norm(a) * torch.linalg.vector_norm(b)))
