"""The latent upsampler on the B200: the tensor-core 3x3 conv kernel against its
CPU emulation, and the FlashLatentUpsampler drop-in against the reference's
own bf16 outputs (golden) and the oracle at the shipped configuration."""
import importlib

import pytest
import torch

from oracle import numerics as onum
from oracle import upsampler as ou
from tests.test_oracle_golden import UPSAMPLER_CASES, upsampler_case
from tests.test_upsampler_cpu import emulate_conv3x3

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def up():
    importlib.import_module("dreamx-creator_b200")
    return importlib.import_module("dreamx-creator_b200.upsampler")


@pytest.mark.parametrize("B,T,H,W,cin,n_src,replicate,shuffle,cout,res,relu", [
    (1, 3, 8, 16, 64, 1, True, 1, 128, False, False),      # one whole tile pair
    (2, 3, 5, 10, 64, 2, True, 1, 64, True, True),         # narrow frames: 8 x 16 blocks
    (2, 2, 6, 10, 128, 2, False, 1, 48, False, True),      # zero memory, a partial N tile
    (1, 3, 4, 130, 64, 1, True, 2, 512, False, True),      # > 128 columns, 4 N tiles, shuffle
    (1, 2, 7, 9, 64, 1, True, 3, 72, False, False),        # shuffle 3, cg 8
    (1, 1, 3, 5, 128, 1, True, 1, 16, True, False),        # an odd number of pixel tiles
])
def test_conv3x3_matches_its_emulation(up, cuda_device, B, T, H, W, cin, n_src, replicate,
                                       shuffle, cout, res, relu):
    ops = up.ops
    g = torch.Generator().manual_seed(H * W + cout)
    F = B * T
    x = torch.randn(F, H, W, cin, generator=g).to(torch.bfloat16)
    w = (torch.randn(cout, n_src * cin, 3, 3, generator=g) * (2.0 / (9 * cin)) ** 0.5)
    w = w.to(torch.bfloat16)
    b = (torch.randn(cout, generator=g) * 0.1).to(torch.bfloat16)
    w2, b2 = ops.conv_weight(w, n_src=n_src, shuffle=shuffle), ops.conv_bias(b, shuffle=shuffle)
    resid = torch.randn(F, H, W, cout, generator=g).to(torch.bfloat16) if res else None
    scale = 0.5 if res else 1.0
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = ops.conv3x3(x.to(cuda_device), w2.to(cuda_device), b2.to(cuda_device),
                      frames_per_clip=T, n_src=n_src, replicate=replicate, shuffle=shuffle,
                      residual=None if resid is None else resid.to(cuda_device),
                      res_scale=scale, relu=relu, status=status)
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0
    ref = emulate_conv3x3(x, w2, b2, T=T, n_src=n_src, replicate=replicate, shuffle=shuffle,
                          residual=resid, res_scale=scale, relu=relu)
    got = out.cpu().double()
    assert got.shape == ref.shape
    # fp32 accumulation in another order than the float64 emulation: values
    # agree to the bit except where a sum sits on a bf16 rounding boundary
    assert onum.rel_fro(got, ref) < 2e-3
    assert float((got == ref).double().mean()) > 0.97


@pytest.mark.parametrize("name", sorted(UPSAMPLER_CASES))
def test_upsampler_matches_the_reference_module(up, cuda_device, golden, name):
    """Against the reference FlashLatentUpsampler's own bf16 output (golden)."""
    sd, x, y, _ = upsampler_case(golden("upsampler"), name)
    kw = UPSAMPLER_CASES[name]
    m = up.FlashLatentUpsampler(sd, in_channels=x.shape[1], out_channels=y.shape[1],
                                mid_channels=sd["blocks.0.conv.2.weight"].shape[0],
                                device=cuda_device, **kw)
    out = m(x.to(cuda_device)).cpu()
    assert out.shape == y.shape and out.dtype == torch.bfloat16
    assert onum.rel_fro(out.double(), y.double()) < 3e-3
    assert onum.cosine(out.double(), y.double()) > 0.99999


def test_upsampler_shipped_configuration(up, cuda_device):
    """configs/latent_upsampler_flash.yaml (48 channels, mid 128, 8 blocks, x2,
    replicate memory) on a 2-frame clip of 18 x 32 latents, seeded weights,
    against the oracle."""
    kw = dict(in_channels=48, out_channels=48, mid_channels=128, num_blocks=8,
              upsample_scale=2)
    sd = up.FlashLatentUpsampler.seeded_state_dict(**kw, seed=4)
    m = up.FlashLatentUpsampler(sd, **kw, memory_init="replicate", residual=False,
                                device=cuda_device)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(1, 48, 2, 18, 32, generator=g).to(torch.bfloat16)
    out = m(x.to(cuda_device)).cpu()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = ou.upsample(sd, x, num_blocks=8, upsample_scale=2, memory_init="replicate")
    assert out.shape == ref.shape == (1, 48, 2, 36, 64)
    assert onum.rel_fro(out.double(), ref) < 5e-3
    assert onum.cosine(out.double(), ref) > 0.9999
