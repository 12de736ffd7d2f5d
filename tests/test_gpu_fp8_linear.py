"""The Fp8Linear drop-in on the GPU: the module swap, the dtype guard and the
call itself against the reference's own ``torch._scaled_mm`` row-wise product
(video_refiner/wan/modules/sr_dit/fp8_linear.py:214-354)."""
import importlib

import pytest
import torch
import torch.nn as nn

from oracle import numerics as onum

pytestmark = pytest.mark.gpu


class _Attn(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.q, self.k, self.v, self.o = (nn.Linear(d, d) for _ in range(4))


class _Block(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.self_attn, self.cross_attn = _Attn(d), _Attn(d)
        self.ffn = nn.Sequential(nn.Linear(d, f), nn.GELU(approximate="tanh"), nn.Linear(f, d))


def _scaled_mm_ref(lin_fp8, x):
    """What the reference Fp8Linear.forward computes for x (fp8_linear.py:282-297),
    with the reference's quantiser restated by the oracle."""
    x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16)
    xq, xs = onum.quantize_rowwise(x2)
    y = torch._scaled_mm(xq, lin_fp8.weight_fp8.t(), scale_a=xs.float(),
                         scale_b=lin_fp8.weight_scale, bias=lin_fp8.bias,
                         out_dtype=torch.bfloat16)
    return y.reshape(*x.shape[:-1], -1)


def test_swap_guard_and_forward(srdit, cuda_device):
    fl = importlib.import_module("dreamx-creator_b200.fp8_linear")
    torch.manual_seed(0)
    d, f = 256, 512
    model = nn.Module()
    model.blocks = nn.ModuleList(_Block(d, f) for _ in range(4))
    model = model.to(cuda_device, torch.bfloat16)
    dense = {n: m.weight.detach().clone() for n, m in model.named_modules()
             if isinstance(m, nn.Linear)}
    names = fl.convert_linears_to_fp8(model, skip_first=1, skip_last=1)
    assert names == [f"blocks.{i}.{t}" for i in (1, 2) for t in fl.TARGETS_ALL]
    assert isinstance(model.blocks[0].ffn[0], nn.Linear)
    assert isinstance(model.blocks[3].self_attn.o, nn.Linear)
    lin = model.blocks[1].self_attn.q
    assert isinstance(lin, fl.Fp8Linear)
    q0, s0 = lin.weight_fp8.clone(), lin.weight_scale.clone()
    # a stray module-wide cast keeps the quantised buffers as they are
    model.to(torch.bfloat16)
    model.float()
    assert lin.weight_fp8.dtype == torch.float8_e4m3fn and lin.weight_scale.dtype == torch.float32
    assert torch.equal(lin.weight_fp8.view(torch.uint8), q0.view(torch.uint8))
    assert torch.equal(lin.weight_scale, s0)
    assert lin.bias.dtype == torch.bfloat16
    assert lin.weight.dtype == torch.float32 and lin.weight.numel() == 0
    # the stored weight is the reference's per-channel quantisation of the dense one
    wq, ws = onum.fp8_linear_weights(dense["blocks.1.self_attn.q"].cpu())
    assert torch.equal(q0.view(torch.uint8).cpu(), wq.view(torch.uint8))
    assert torch.equal(s0.reshape(-1).cpu(), ws)
    # 3-D input through the module vs the exact row-wise scaled product (the
    # oracle: fp64 accumulation, one rounding to bf16) and vs the reference's own
    # _scaled_mm call. At these small sizes cuBLASLt's bf16 output is itself up
    # to a few 1e-3 away from the exact product, so the module must be within
    # 1e-3 of the exact product and no further from cuBLASLt than twice
    # cuBLASLt's own error (BASELINE's sizes: tests/test_gpu_config2.py, 1e-3).
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(2, 37, d, generator=g, device=cuda_device).to(torch.bfloat16)
    for name in ("self_attn.q", "cross_attn.o", "ffn.0", "ffn.2"):
        mod = model.blocks[2].get_submodule(name)
        xin = x if mod.in_features == d else torch.randn(2, 37, mod.in_features, generator=g,
                                                         device=cuda_device).to(torch.bfloat16)
        y = mod(xin)
        assert y.shape == (2, 37, mod.out_features) and y.dtype == torch.bfloat16
        exact = onum.fp8_linear(xin.cpu(), mod.weight_fp8.cpu(), mod.weight_scale.cpu(),
                                mod.bias.cpu())
        ref = _scaled_mm_ref(mod, xin)
        err_exact = onum.rel_fro(y.float().cpu(), exact.float())
        err_ref_exact = onum.rel_fro(ref.float().cpu(), exact.float())
        assert err_exact <= 1e-3, (name, err_exact, err_ref_exact)
        assert onum.rel_fro(y.float(), ref.float()) <= max(1e-3, 2 * err_ref_exact), name
    # an fp32 input comes back fp32 (the product is computed from its bf16 rounding)
    y32 = lin(x.float())
    assert y32.dtype == torch.float32
    assert torch.equal(y32, lin(x).float())
    # the whole block FFN runs through two swapped Linears
    h = model.blocks[1].ffn(x)
    ref_h = model.blocks[1].ffn[2](model.blocks[1].ffn[1](model.blocks[1].ffn[0](x)))
    assert torch.equal(h, ref_h)
