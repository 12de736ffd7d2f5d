"""The Wan2.2 VAE decode on the B200: srdit_conv3d in each of its forms and
srdit_rms_silu against their emulations / the oracle, and the whole decoder
against the reference WanVAE_.decode (golden) and the oracle."""
import importlib

import pytest
import torch

from oracle import numerics as onum
from oracle import vae as ov
from tests.golden_cases import vae_state_dict
from tests.cpu_ops import emulate_conv3d

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pkg():
    importlib.import_module("dreamx-creator_b200")
    return (importlib.import_module("dreamx-creator_b200.ops"),
            importlib.import_module("dreamx-creator_b200.vae"))


def _rand(shape, g, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("Fo,H,W,cin,cout,kt,kh,shuffle_t,res", [
    (2, 5, 10, 64, 64, 3, 3, 1, True),       # a causal 3x3x3 conv with the residual add
    (3, 4, 130, 128, 48, 3, 3, 1, False),    # > 128 columns, a partial N tile
    (2, 3, 8, 64, 128, 3, 1, 2, False),      # the time_conv: 3x1x1, frames interleaved
    (1, 6, 7, 128, 192, 1, 1, 1, True),      # 1x1 (shortcut / qkv / proj), 2 N tiles
    (1, 8, 16, 64, 16, 3, 3, 1, False),      # the head (12 channels padded to 16)
])
def test_conv3d_matches_its_emulation(pkg, cuda_device, Fo, H, W, cin, cout, kt, kh, shuffle_t,
                                      res):
    ops, _ = pkg
    g = torch.Generator().manual_seed(Fo * 100 + W + cout)
    x = _rand((Fo + kt - 1, H, W, cin), g)
    w = _rand((cout, cin, kt, kh, kh), g, (1.0 / (cin * kt * kh * kh)) ** 0.5)
    b = (torch.randn(cout, generator=g) * 0.1).float()
    w2 = ops.conv3d_weight(w)
    r = _rand((Fo, H, W, cout), g) if res else None
    st = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = ops.conv3d(x.to(cuda_device), w2.to(cuda_device), b.to(cuda_device), kt=kt, kh=kh,
                     shuffle_t=shuffle_t, residual=None if r is None else r.to(cuda_device),
                     status=st)
    torch.cuda.synchronize(cuda_device)
    assert int(st.item()) == 0
    ref = emulate_conv3d(x, w2, b, kt=kt, kh=kh, shuffle_t=shuffle_t, residual=r)
    got = out.cpu().double()
    assert got.shape == ref.shape
    assert onum.rel_fro(got, ref) < 2e-3
    assert float((got == ref).double().mean()) > 0.97


def test_up2_phase_launches(pkg, cuda_device):
    """Four phase launches = nearest 2x upsample + 3x3 conv, with the residual."""
    ops, _ = pkg
    g = torch.Generator().manual_seed(8)
    T, H, W, C = 2, 5, 9, 128
    x = _rand((T, H, W, C), g)
    w = _rand((C, C, 3, 3), g, (1.0 / (9 * C)) ** 0.5)
    b = (torch.randn(C, generator=g) * 0.1).float()
    r = _rand((T, 2 * H, 2 * W, C), g)
    w2 = ops.conv3d_weight(w)
    out = torch.full((T, 2 * H, 2 * W, C), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    for ph in range(4):
        ops.conv3d(x.to(cuda_device), w2.to(cuda_device), b.to(cuda_device), kt=1, kh=3,
                   up2_phase=ph, out=out, residual=r.to(cuda_device))
    got = out.cpu().double()
    assert not torch.isnan(got).any()            # every sub-pixel written
    ref = sum(emulate_conv3d(x, w2, b, kt=1, kh=3, up2_phase=ph, residual=r) for ph in range(4))
    assert onum.rel_fro(got, ref) < 2e-3
    assert float((got == ref).double().mean()) > 0.97


@pytest.mark.parametrize("C", [64, 256, 1024])
def test_rms_silu_matches_the_oracle(pkg, cuda_device, C):
    ops, _ = pkg
    g = torch.Generator().manual_seed(C)
    x = _rand((2, 5, 7, C), g, 3.0)
    x[0, 0, 0] = 0                                 # a zero pixel: the eps clamp
    gamma = _rand((C,), g, 0.3) + 1
    for silu in (True, False):
        got = ops.rms_silu(x.to(cuda_device), gamma.to(cuda_device), silu=silu).cpu().double()
        ref = ov.rms_norm(x.double().permute(3, 0, 1, 2), gamma.double())
        if silu:
            ref = ov.silu(ref)
        ref = ref.permute(1, 2, 3, 0)
        assert torch.isfinite(got).all()
        assert float((got == ref).double().mean()) > 0.99
        assert onum.rel_fro(got, ref) < 1e-3


def test_decode_matches_the_reference(pkg, cuda_device, golden):
    """The whole decode (3 latent frames -> 9 frames, Wan2.2 structure at width
    64) against the reference's bf16 WanVAE_.decode and the oracle: the same
    distance as the bf16 reference keeps from fp32 (rounding noise amplified
    through ~30 convs, about 1.3% here), cosine >= 0.9995."""
    _, vae = pkg
    g = golden("vae")
    sd = vae_state_dict(g)
    z = torch.from_numpy(g["z"]).view(torch.bfloat16)
    mean, std = torch.from_numpy(g["mean"]), torch.from_numpy(g["std"])
    y = torch.from_numpy(g["y"]).view(torch.bfloat16).double()
    y32 = torch.from_numpy(g["y32"]).double()
    d = vae.Wan22VAEDecoder(sd, dim=64, device=cuda_device)
    out = d.decode(z.to(cuda_device), mean, std, clamp=False).cpu().double()
    assert out.shape == y.shape == (3, 9, 64, 96)
    for ref in (y, y32):
        assert onum.rel_fro(out, ref) < 3e-2
        assert onum.cosine(out, ref) > 0.9995
    # clamped as the pipeline's wrapper returns it
    outc = d.decode(z.to(cuda_device), mean, std).cpu()
    assert outc.min() >= -1 and outc.max() <= 1
    assert torch.equal(outc, out.float().clamp(-1, 1))


@pytest.mark.parametrize("cin,cout,ft,shift", [(128, 128, 2, 0), (128, 128, 2, 1),
                                               (256, 128, 1, 0)])
def test_dup_up_gathered_in_the_epilogue(pkg, cuda_device, cin, cout, ft, shift):
    """The phase launches' DupUp3D residual, gathered from the block input in the
    epilogue, equals the materialised DupUp3D tensor added as a residual."""
    ops, vae = pkg
    g = torch.Generator().manual_seed(cin + 10 * ft + shift)
    Tb, H, W = 2, 3, 5
    Tc = Tb * ft - shift
    xb = _rand((Tb, H, W, cin), g).to(cuda_device)
    xc = _rand((Tc, H, W, cout), g).to(cuda_device)
    w2 = ops.conv3d_weight(_rand((cout, cout, 3, 3), g, (1.0 / (9 * cout)) ** 0.5)).to(cuda_device)
    b = (torch.randn(cout, generator=g) * 0.1).float().to(cuda_device)
    fused = torch.empty(Tc, 2 * H, 2 * W, cout, dtype=torch.bfloat16, device=cuda_device)
    mat = torch.empty_like(fused)
    res = vae._dup_up(xb, cout, ft, 2, shift > 0)
    for ph in range(4):
        ops.conv3d(xc, w2, b, kt=1, kh=3, up2_phase=ph, out=fused, dup=(xb, ft, shift))
        ops.conv3d(xc, w2, b, kt=1, kh=3, up2_phase=ph, out=mat, residual=res)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(fused, mat)


def test_decode_at_full_width(pkg, cuda_device):
    """The shipped decoder's widths (dec_dim 256: 1024-channel layers, 8 output
    tiles, 27 x 16 K slices per tap set) on a small latent (2 frames of 2 x 3,
    seeded weights) against the oracle."""
    _, vae = pkg
    sd = vae.Wan22VAEDecoder.seeded_state_dict(seed=5)
    g = torch.Generator().manual_seed(1)
    z = torch.randn(48, 2, 2, 3, generator=g).to(torch.bfloat16)
    mean, std = 0.1 * torch.randn(48, generator=g), 0.5 + torch.rand(48, generator=g)
    d = vae.Wan22VAEDecoder(sd, device=cuda_device)
    out = d.decode(z.to(cuda_device), mean, std, clamp=False).cpu().double()
    ref = ov.Decoder(sd).decode(z, mean, std)
    assert out.shape == ref.shape == (3, 5, 32, 48)
    assert onum.rel_fro(out, ref) < 3e-2
    assert onum.cosine(out, ref) > 0.9995
