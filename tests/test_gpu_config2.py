"""BASELINE config 2 at its own sizes: every (M, K, N) of the fp8 Linear sweep.

M in {6912, 20736, 41472} tokens x (K, N) in {(3072, 3072), (3072, 9216) fused
q|k|v, (3072, 14336) ffn.0, (14336, 3072) ffn.2}. Activations bf16 N(0,1) with
0.1% outliers x20, quantised per token to e4m3; weights N(0, 0.02) quantised per
output channel; bias N(0, 0.01); bf16 out. The B200 GEMM is compared with the
reference's own GPU call on the same operands -- cuBLASLt row-wise
``torch._scaled_mm(xq, w_fp8.t(), scale_a, scale_b, bias, out_dtype=bf16)``
(video_refiner/wan/modules/sr_dit/fp8_linear.py:291-294) -- over the whole
output, and with the CPU oracle (dequantised product, fp64 accumulation) on
96 rows spread over M. Tolerance: relative Frobenius error <= 1e-3.
"""
import pytest
import torch

from oracle import numerics as onum

pytestmark = pytest.mark.gpu

SHAPES = [(M, N, K) for M in (6912, 20736, 41472)
          for (K, N) in ((3072, 3072), (3072, 9216), (3072, 14336), (14336, 3072))]


@pytest.mark.parametrize("M,N,K", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_config2_gemm_matches_scaled_mm_and_oracle(srdit, cuda_device, M, N, K):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(M * 31 + N * 7 + K)
    a = torch.randn(M, K, generator=g, device=dev)
    a = torch.where(torch.rand(M, K, generator=g, device=dev) < 1e-3, a * 20, a)
    a = a.to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g, device=dev) * 0.01).to(torch.bfloat16)
    aq, as_ = srdit.ops.quant_rowwise(a)
    wq, ws = srdit.fp8_linear.quantize_weight(w)
    out = srdit.ops.fp8_gemm(aq, as_, wq, ws, bias)
    ref = torch._scaled_mm(aq, wq.t(), scale_a=as_.view(-1, 1), scale_b=ws.view(1, -1),
                           bias=bias, out_dtype=torch.bfloat16)
    err = onum.rel_fro(out.float(), ref.float())
    assert err <= 1e-3, err
    del ref
    rows = torch.linspace(0, M - 1, 96).round().long()
    rows_d = rows.to(dev)
    ora = onum.fp8_linear(a[rows_d].cpu(), wq.cpu(), ws.cpu(), bias.cpu())
    err_o = onum.rel_fro(out[rows_d].cpu().float(), ora.float())
    assert err_o <= 1e-3, err_o
