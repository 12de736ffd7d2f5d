"""Host-side logic of the Fp8Linear drop-in (no GPU): weight preparation, the
dtype-preserving module conversions and the module swap of
convert_linears_to_fp8 (video_refiner/wan/modules/sr_dit/fp8_linear.py:214-354).
The GEMM itself runs only on the GPU (tests/test_gpu_fp8_linear.py)."""
import importlib

import pytest
import torch
import torch.nn as nn

from oracle import numerics as onum


@pytest.fixture(scope="module")
def fl(srdit):
    return importlib.import_module("dreamx-creator_b200.fp8_linear")


class _Attn(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.q, self.k, self.v, self.o = (nn.Linear(d, d) for _ in range(4))


class _Block(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.self_attn, self.cross_attn = _Attn(d), _Attn(d)
        self.ffn = nn.Sequential(nn.Linear(d, f), nn.GELU(approximate="tanh"), nn.Linear(f, d))


class _Model(nn.Module):
    def __init__(self, n=4, d=64, f=128):
        super().__init__()
        torch.manual_seed(0)
        self.blocks = nn.ModuleList(_Block(d, f) for _ in range(n))
        self.head = nn.Linear(d, 8)


def test_weight_quantisation_is_the_reference_rule(fl):
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(96, 160, generator=g) * 0.02).to(torch.bfloat16)
    w[3] = 0
    q, s = fl.quantize_weight(w)
    qo, so = onum.fp8_linear_weights(w)
    assert torch.equal(q.view(torch.uint8), qo.view(torch.uint8))
    assert torch.equal(s, so)


def test_module_casts_keep_fp8_buffers(fl):
    lin = nn.Linear(64, 32).to(torch.bfloat16)
    m = fl.Fp8Linear.from_linear(lin)
    q0, s0, b0 = m.weight_fp8.clone(), m.weight_scale.clone(), m.bias.clone()
    assert (q0.dtype, s0.dtype, b0.dtype) == (torch.float8_e4m3fn, torch.float32, torch.bfloat16)
    assert s0.shape == (1, 32) and m.weight.numel() == 0 and m.weight.dtype == torch.bfloat16
    for cast in (lambda t: t.to(torch.bfloat16), lambda t: t.float(), lambda t: t.half(),
                 lambda t: t.to("cpu", torch.float64)):
        out = cast(m)
        assert out is m
        assert m.weight_fp8.dtype == torch.float8_e4m3fn
        assert torch.equal(m.weight_fp8.view(torch.uint8), q0.view(torch.uint8))
        assert m.weight_scale.dtype == torch.float32 and torch.equal(m.weight_scale, s0)
        assert m.bias.dtype == torch.bfloat16 and torch.equal(m.bias, b0)
    # the stand-in follows the casts (callers read .weight.dtype)
    assert m.weight.dtype == torch.float64
    with pytest.raises(ValueError):
        fl.Fp8Linear(torch.zeros(4, 4, 4))


def test_no_bias_and_fp32_bias_narrowed(fl):
    m = fl.Fp8Linear(torch.randn(16, 32), None)
    assert m.bias is None
    m2 = fl.Fp8Linear(torch.randn(16, 32), torch.randn(16))
    assert m2.bias.dtype == torch.bfloat16


def test_convert_needs_cuda(fl, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(Exception, match="CUDA"):
        fl.convert_linears_to_fp8(_Model())


def test_convert_swaps_targets_with_skips(fl, monkeypatch):
    """The swap itself (construction runs on CPU tensors): blocks 1..2 of 4
    converted with skip_first=1 / skip_last=1, every target path, nothing else;
    a second call converts nothing."""
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    model = _Model()
    names = fl.convert_linears_to_fp8(model, skip_first=1, skip_last=1)
    assert names == [f"blocks.{i}.{t}" for i in (1, 2) for t in fl.TARGETS_ALL]
    for i, blk in enumerate(model.blocks):
        for t in fl.TARGETS_ALL:
            mod = blk.get_submodule(t)
            assert isinstance(mod, fl.Fp8Linear) == (i in (1, 2)), (i, t)
    assert isinstance(model.blocks[1].ffn[1], nn.GELU)     # non-targets untouched
    assert isinstance(model.head, nn.Linear)
    assert fl.convert_linears_to_fp8(model, skip_first=1, skip_last=1) == []
    ffn_only = _Model()
    got = fl.convert_linears_to_fp8(ffn_only, targets=fl.TARGETS_FFN)
    assert got == [f"blocks.{i}.ffn.{j}" for i in range(4) for j in (0, 2)]
    assert fl.convert_linears_to_fp8(nn.Linear(4, 4)) == []  # no blocks: nothing to do
