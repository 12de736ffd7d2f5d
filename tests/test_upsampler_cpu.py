"""The latent upsampler's host side, without a GPU: the conv kernel's weight
layout and index arithmetic (emulated here exactly as csrc/conv.cu addresses
its operands) against torch's conv2d + PixelShuffle, and the drop-in class's
parameter names and argument checks against the reference module's."""
import importlib

import pytest
import torch

from tests.test_oracle_golden import UPSAMPLER_CASES


@pytest.fixture(scope="module")
def up():
    importlib.import_module("dreamx-creator_b200")
    return importlib.import_module("dreamx-creator_b200.upsampler")


@pytest.fixture(scope="module")
def ops():
    importlib.import_module("dreamx-creator_b200")
    return importlib.import_module("dreamx-creator_b200.ops")


def emulate_conv3x3(x, w2, bias, *, T, n_src, replicate, shuffle, residual=None,
                    res_scale=1.0, relu=False):
    """srdit_conv3x3's arithmetic in float64: source s of output frame f is frame
    f (s = 0) or the clip's previous frame (s = 1; the first frame: itself or
    zeros), tap (ky, kx) reads pixel (h + ky - 1, w + kx - 1) (zeros outside), K
    index (s * 9 + ky * 3 + kx) * cin + c; shuffled stores as the kernel's."""
    F, H, W, cin = x.shape
    cout = w2.shape[0]
    xp = torch.nn.functional.pad(x.double(), (0, 0, 1, 1, 1, 1))   # [F, H+2, W+2, cin]
    cols = []
    for s in range(n_src):
        src = xp
        if s == 1:
            prev = torch.zeros_like(xp)
            for f in range(F):
                if f % T > 0:
                    prev[f] = xp[f - 1]
                elif replicate:
                    prev[f] = xp[f]
            src = prev
        for ky in range(3):
            for kx in range(3):
                cols.append(src[:, ky:ky + H, kx:kx + W, :])
    a = torch.cat(cols, dim=-1)                                      # [F, H, W, K]
    y = a @ w2.double().t() + bias.double()
    y = y.to(torch.float32).to(torch.bfloat16).double()
    if residual is not None:
        if res_scale != 1.0:
            y = (y * res_scale).to(torch.float32).to(torch.bfloat16).double()
        y = (residual.double() + y).to(torch.float32).to(torch.bfloat16).double()
    if relu:
        y = y.clamp_min(0)
    r = shuffle
    if r == 1:
        return y
    cg = cout // (r * r)
    out = torch.empty(F, r * H, r * W, cg, dtype=torch.float64)
    for n in range(cout):
        g, c = divmod(n, cg)
        i, j = divmod(g, r)
        out[:, i::r, j::r, c] = y[..., n]
    return out


@pytest.mark.parametrize("cin,cin_pad,n_src,replicate,shuffle,cout", [
    (16, 64, 1, True, 2, 64), (64, 64, 2, True, 1, 64), (64, 64, 2, False, 1, 48),
    (48, 64, 1, True, 3, 72), (128, 128, 1, True, 1, 16)])
def test_kernel_layout_reproduces_conv_and_pixel_shuffle(ops, cin, cin_pad, n_src, replicate,
                                                         shuffle, cout):
    g = torch.Generator().manual_seed(cin + cout + shuffle)
    B, T, H, W = 2, 3, 5, 7
    x = torch.randn(B * T, cin, H, W, generator=g).to(torch.bfloat16)
    w = (torch.randn(cout, n_src * cin, 3, 3, generator=g) * 0.1).to(torch.bfloat16)
    b = (torch.randn(cout, generator=g) * 0.1).to(torch.bfloat16)
    # torch: conv over cat([x, past]) then PixelShuffle, NCHW
    xin = x.double()
    if n_src == 2:
        xb = xin.reshape(B, T, cin, H, W)
        first = xb[:, :1] if replicate else torch.zeros_like(xb[:, :1])
        past = torch.cat([first, xb[:, :-1]], 1).reshape(xin.shape)
        xin = torch.cat([xin, past], 1)
    ref = torch.nn.functional.conv2d(xin, w.double(), b.double(), padding=1)
    ref = ref.to(torch.float32).to(torch.bfloat16).double()
    if shuffle > 1:
        ref = torch.nn.functional.pixel_shuffle(ref, shuffle)
    ref = ref.permute(0, 2, 3, 1)
    # the kernel's operands: channels-last frames padded to cin_pad, K-major weight
    xl = torch.nn.functional.pad(x.permute(0, 2, 3, 1), (0, cin_pad - cin))
    w2 = ops.conv_weight(w, n_src=n_src, cin_pad=cin_pad, shuffle=shuffle)
    b2 = ops.conv_bias(b, shuffle=shuffle)
    assert w2.shape == (cout, n_src * 9 * cin_pad) and w2.dtype == torch.bfloat16
    got = emulate_conv3x3(xl, w2, b2, T=T, n_src=n_src, replicate=replicate, shuffle=shuffle)
    assert got.shape == ref.shape
    # the same products summed in another order, one bf16 rounding
    assert (got - ref).abs().max() <= 2 ** -7 * ref.abs().max()
    assert float((got == ref).double().mean()) > 0.9


def test_seeded_state_dict_has_the_reference_parameters(up, golden):
    g = golden("upsampler")
    for name, kw in (("x2_replicate", dict(in_channels=16, mid_channels=64, num_blocks=2,
                                           upsample_scale=2)),
                     ("x4_residual", dict(in_channels=16, mid_channels=64, num_blocks=1,
                                          upsample_scale=4, residual=True))):
        sd = up.FlashLatentUpsampler.seeded_state_dict(**kw)
        pre = name + ".sd."
        ref = {k[len(pre):]: v.shape for k, v in g.items() if k.startswith(pre)}
        assert {k: tuple(v.shape) for k, v in sd.items()} == ref, name


def test_constructor_checks(up):
    sd = up.FlashLatentUpsampler.seeded_state_dict(in_channels=16, mid_channels=64,
                                                    num_blocks=1)
    kw = dict(in_channels=16, mid_channels=64, num_blocks=1, device="cpu")
    with pytest.raises(ValueError):
        up.FlashLatentUpsampler(sd, **{**kw, "memory_init": "ema"})
    with pytest.raises(ValueError):
        up.FlashLatentUpsampler(sd, **{**kw, "num_blocks": 0})
    with pytest.raises(up._lib.SrditError, match="ReLU"):
        up.FlashLatentUpsampler(sd, **{**kw, "activation": "silu"})
    with pytest.raises(up._lib.SrditError, match="ema_alpha"):
        up.FlashLatentUpsampler(sd, **{**kw, "ema_alpha": 0.5})
    m = up.FlashLatentUpsampler(sd, **kw)
    # the conv weights are already in the kernel's layout; nothing runs without a GPU
    assert m.head[0].w.shape == (64 * 4, 9 * 64) and m.blocks[0][0].n_src == 2
    with pytest.raises(up._lib.SrditError):
        m(torch.zeros(1, 16, 2, 4, 4, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        m(torch.zeros(1, 8, 2, 4, 4))
    assert m.flops(T=2, H=4, W=4) == 2 * 2 * (
        16 * 256 * 9 * 16 + 64 * (64 * 9 * 128 + 2 * 64 * 9 * 64 + 16 * 9 * 64))


def test_oracle_cases_are_covered():
    assert set(UPSAMPLER_CASES) == {"x2_replicate", "x4_residual"}
