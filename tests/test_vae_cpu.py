"""The VAE decode's host side, without a GPU: srdit_conv3d's operand layout and
index arithmetic (emulated as csrc/conv.cu addresses them) against torch's
conv3d / the upsample-then-conv / the time_conv frame interleave, DupUp3D on
channels-last frames against the oracle's, and the decoder built from the
reference's state dict."""
import importlib

import pytest
import torch

from oracle import vae as ov
from tests.cpu_ops import emulate_conv3d


@pytest.fixture(scope="module")
def pkg():
    importlib.import_module("dreamx-creator_b200")
    return (importlib.import_module("dreamx-creator_b200.ops"),
            importlib.import_module("dreamx-creator_b200.vae"))


def _rand(shape, g, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("kt,kh,cin,cout", [(3, 3, 64, 64), (3, 1, 64, 128), (1, 1, 128, 64)])
def test_conv3d_layout_is_a_causal_conv(pkg, kt, kh, cin, cout):
    ops, _ = pkg
    g = torch.Generator().manual_seed(kt * 10 + kh + cin)
    T, H, W = 3, 5, 6
    x = _rand((cin, T, H, W), g)
    w = _rand((cout, cin, kt, kh, kh), g, (1.0 / (cin * kt * kh * kh)) ** 0.5)
    b = _rand((cout,), g, 0.1)
    cache = _rand((cin, 2, H, W), g) if kt == 3 else None
    ref = ov.causal_conv(x.double(), w, b, cache.double() if cache is not None else None)
    hist = x.permute(1, 2, 3, 0)
    if kt == 3:
        hist = torch.cat([cache.permute(1, 2, 3, 0), hist])
    w2 = ops.conv3d_weight(w)
    got = emulate_conv3d(hist, w2, b.float(), kt=kt, kh=kh)
    assert got.shape == (T, H, W, cout)
    ref = ref.permute(1, 2, 3, 0)
    assert (got - ref).abs().max() <= 2 ** -7 * ref.abs().max()
    assert float((got == ref).double().mean()) > 0.9


def test_up2_phases_are_upsample_then_conv(pkg):
    """The four phase launches together are nearest 2x + Conv2d(3x3, pad 1)."""
    ops, _ = pkg
    g = torch.Generator().manual_seed(5)
    T, H, W, C = 2, 4, 5, 64
    x = _rand((T, H, W, C), g)
    w = _rand((C, C, 3, 3), g, (1.0 / (9 * C)) ** 0.5)
    b = _rand((C,), g, 0.1)
    res = _rand((T, 2 * H, 2 * W, C), g)
    up = x.double().repeat_interleave(2, 1).repeat_interleave(2, 2)
    ref = torch.nn.functional.conv2d(up.permute(0, 3, 1, 2), w.double(), b.double(), padding=1)
    ref = ref.to(torch.float32).to(torch.bfloat16).double().permute(0, 2, 3, 1)
    ref = (res.double() + ref).to(torch.float32).to(torch.bfloat16).double()
    w2 = ops.conv3d_weight(w)
    got = sum(emulate_conv3d(x, w2, b.float(), kt=1, kh=3, up2_phase=ph, residual=res)
              for ph in range(4))
    assert (got - ref).abs().max() <= 2 ** -7 * ref.abs().max()
    assert float((got == ref).double().mean()) > 0.9


def test_time_conv_interleave(pkg):
    """shuffle_t = 2 stores channel half k of output frame t as frame 2 t + k: the
    reshape(b, 2, c, t, h, w) / stack of Resample's upsample3d."""
    ops, _ = pkg
    g = torch.Generator().manual_seed(6)
    T, H, W, C = 2, 3, 4, 64
    x = _rand((C, T, H, W), g)
    w = _rand((2 * C, C, 3, 1, 1), g, (1.0 / (3 * C)) ** 0.5)
    b = _rand((2 * C,), g, 0.1)
    y = ov.causal_conv(x.double(), w, b, None).reshape(2, C, T, H, W)
    ref = torch.stack([y[0], y[1]], 2).reshape(C, 2 * T, H, W).permute(1, 2, 3, 0)
    hist = torch.cat([torch.zeros(2, H, W, C, dtype=torch.bfloat16), x.permute(1, 2, 3, 0)])
    got = emulate_conv3d(hist, ops.conv3d_weight(w), b.float(), kt=3, kh=1, shuffle_t=2)
    assert got.shape == ref.shape
    assert (got - ref).abs().max() <= 2 ** -7 * ref.abs().max()


@pytest.mark.parametrize("cin,cout,ft,first", [(128, 128, 2, False), (128, 128, 2, True),
                                               (128, 64, 1, False)])
def test_dup_up_matches_the_oracle(pkg, cin, cout, ft, first):
    _, vae = pkg
    g = torch.Generator().manual_seed(cin + ft)
    x = _rand((cin, 2, 3, 4), g)
    ref = ov.Decoder._dup_up(x.double(), cout, ft, 2, first).permute(1, 2, 3, 0)
    got = vae._dup_up(x.permute(1, 2, 3, 0).contiguous(), cout, ft, 2, first)
    assert torch.equal(got.double(), ref)


def test_decoder_builds_from_the_reference_state_dict(pkg, golden):
    from tests.golden_cases import vae_state_dict
    _, vae = pkg
    sd = vae_state_dict(golden("vae"))
    d = vae.Wan22VAEDecoder(sd, dim=64, device="cpu")
    assert [c.kt for c in (d.conv1, d.head)] == [3, 3] and d.head.cout_pad == 16
    assert [len(u.res) for u in d.ups] == [3, 3, 3, 3]
    assert [u.resample.mode if u.resample else None for u in d.ups] == \
        ["upsample3d", "upsample3d", "upsample2d", None]
    assert d.ups[2].res[0].short is not None and d.ups[0].res[0].short is None
    with pytest.raises(importlib.import_module("dreamx-creator_b200._lib").SrditError):
        d.decode(torch.zeros(48, 1, 4, 6), torch.zeros(48), torch.ones(48))


def test_param_shapes_are_the_reference_decoders(pkg, golden):
    """The decoder's parameter names and shapes (used for seeded weights) are the
    reference WanVAE_ state dict's, at the golden's width."""
    _, vae = pkg
    g = golden("vae")
    ref = {str(n): tuple(int(v) for v in shp[:int(nd)])
           for n, shp, nd in zip(g["param_names"], g["param_shapes"], g["param_ndims"])}
    assert vae.Wan22VAEDecoder.param_shapes(dim=64) == ref
    sd = vae.Wan22VAEDecoder.seeded_state_dict(dim=64)
    d = vae.Wan22VAEDecoder(sd, dim=64, device="cpu")
    # 3 latent frames of 4 x 6: the head alone is 27 taps x 64 -> 12 on 9 frames
    assert d.flops(3, 4, 6) > 2 * 9 * 32 * 48 * 12 * 64 * 27


def test_decoder_host_logic_on_the_cpu_double(pkg, golden, monkeypatch):
    """The decoder's orchestration -- the history buffers and their shifts, the
    skipped first time conv, the phase launches and their DupUp3D source, the
    attention, unpatchify -- run with the CPU double of its kernels (their
    emulations, float64 sums with the kernels' roundings) and the oracle's
    attention, reproduces the oracle's bf16 decode of the golden case."""
    from oracle import numerics as onum
    from tests import cpu_ops
    from tests.golden_cases import vae_state_dict
    _, vae = pkg
    monkeypatch.setattr(vae, "ops", cpu_ops)
    monkeypatch.setattr(vae, "attend", cpu_ops.vae_attend)
    g = golden("vae")
    sd = vae_state_dict(g)
    z = torch.from_numpy(g["z"]).view(torch.bfloat16)
    mean, std = torch.from_numpy(g["mean"]), torch.from_numpy(g["std"])
    d = vae.Wan22VAEDecoder(sd, dim=64, device="cpu")
    out = d.decode(z, mean, std, clamp=False).double()
    ref = ov.Decoder(sd).decode(z, mean, std)
    assert out.shape == ref.shape
    assert onum.rel_fro(out, ref) < 1e-3
    assert float((out == ref).double().mean()) > 0.95
