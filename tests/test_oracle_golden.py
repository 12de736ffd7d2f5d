"""Pin the CPU oracle against golden vectors produced by the reference itself."""
import numpy as np
import pytest
import torch

from oracle import blockgrid as obg
from oracle import numerics as onum
from oracle import winattn as owa
from tests.golden_cases import PLAN_NAMES, spec_from_golden


def bf16(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16)


@pytest.mark.parametrize("name", PLAN_NAMES)
def test_oracle_plan_matches_reference(golden, name):
    g = golden("plans")
    spec, mode = spec_from_golden(g, name, obg.Spec)
    plan = obg.build_plan(spec, mode)
    np.testing.assert_array_equal(plan["params"], g[f"{name}.params"])
    meta = [plan["n_w"], plan["block_m"], plan["m_tiles"], plan["block_n"], plan["hr_base"],
            plan["p_stride"]]
    np.testing.assert_array_equal(meta, g[f"{name}.meta"])


@pytest.mark.parametrize("name", PLAN_NAMES)
def test_oracle_plan_partitions_queries(golden, name):
    g = golden("plans")
    spec, mode = spec_from_golden(g, name, obg.Spec)
    plan = obg.build_plan(spec, mode)
    cnt = owa.coverage(plan, spec.f_cur, spec.h, spec.w)
    assert (cnt == 1).all()


def test_oracle_quant_bit_exact(golden):
    g = golden("quant")
    q, s = onum.quantize_rowwise(bf16(g["x"]))
    np.testing.assert_array_equal(q.view(torch.uint8).numpy(), g["q"])
    np.testing.assert_array_equal(s.numpy(), g["s"])


def test_oracle_norms_bit_exact(golden):
    g = golden("norms")
    x = bf16(g["x"])
    np.testing.assert_array_equal(onum.layer_norm(x).view(torch.int16).numpy(), g["ln"])
    y = onum.layer_norm(x, weight=bf16(g["lna_w"]), bias=bf16(g["lna_b"]))
    np.testing.assert_array_equal(y.view(torch.int16).numpy(), g["lna"])
    y = onum.rms_norm(x, bf16(g["rms_w"]))
    np.testing.assert_array_equal(y.view(torch.int16).numpy(), g["rms"])


def test_oracle_rope_bit_exact(golden):
    g = golden("rope")
    freqs = onum.rope_freqs()
    np.testing.assert_array_equal(freqs.real.numpy()[:16], g["freqs_re"])
    np.testing.assert_array_equal(freqs.imag.numpy()[:16], g["freqs_im"])
    y = onum.rope_apply(bf16(g["x"]), (2, 5, 7), freqs, t_offset=3)
    np.testing.assert_array_equal(y.view(torch.int16).numpy(), g["y"])
    yf = onum.rope_apply(torch.from_numpy(g["xf"]), (2, 5, 7), freqs, t_offset=0)
    np.testing.assert_array_equal(yf.numpy(), g["yf"])


@pytest.mark.parametrize("tag,bhw,rhw", [("cfg1_8x8_r0", (8, 8), (0, 0)),
                                         ("cfg1_4x4_r3", (4, 4), (3, 3))])
def test_oracle_window_attention_config1(golden, tag, bhw, rhw):
    """the reference's sdpa path, fp32, seed 0."""
    g = golden("winattn")
    from tests.golden_cases import config1_inputs
    qr, kr, v = config1_inputs()
    spec = obg.make_spec(3, 3, 18, 32, block_t=3, block_hw=bhw, block_radius_hw=rhw)
    plan = obg.build_plan(spec)
    out = owa.run_plan(qr, kr, v, plan, f_cur=3, h=18, w=32, dtype=torch.float64)
    np.testing.assert_allclose(out[:, 0].numpy(), g[f"{tag}.out_h0"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(out[::97].numpy(), g[f"{tag}.rows"], rtol=0, atol=2e-5)
    sums = [float(out.sum()), float(out.abs().sum()), float((out ** 2).sum())]
    np.testing.assert_allclose(sums, g[f"{tag}.sum"], rtol=1e-6)


@pytest.mark.parametrize("tag", ["none", "frame", "chunk"])
def test_oracle_window_attention_streaming(golden, tag):
    """KV cache + LQ anchor (frame / chunk align), small grid, 2 heads."""
    g = golden("winattn")
    from tests.golden_cases import stream_inputs
    ins = stream_inputs()
    np.testing.assert_allclose([float(t.double().sum()) for t in ins.values()],
                               g["stream.input_sums"], rtol=1e-12)
    f_cur, h, w = 3, 8, 12
    anchor = None if tag == "none" else tag
    spec = obg.make_spec(3, 6, h, w, block_t=3, block_hw=(4, 4), block_radius_hw=(1, 1),
                         streaming=True)
    plan = obg.build_plan(spec, anchor)
    k_full = torch.cat([ins["ck"], ins["k"]])
    v_full = torch.cat([ins["cv"], ins["v"]])
    if anchor is not None:
        k_full = torch.cat([ins["ak"], k_full])
        v_full = torch.cat([ins["av"], v_full])
    out = owa.run_plan(ins["q"], k_full, v_full, plan, f_cur=f_cur, h=h, w=w)
    np.testing.assert_allclose(out.numpy(), g[f"stream.{tag}.out"], rtol=0, atol=2e-5)


def _block_golden(golden):
    g = golden("block")
    dim, ffn, heads, f_cur, h, w, ctx_len, f_cache = (int(x) for x in g["dims"])
    wts = {}
    for k, v in g.items():
        if k.startswith("w."):
            t = torch.from_numpy(v)
            wts[k[2:]] = t.view(torch.bfloat16) if t.dtype == torch.int16 else t
    t = {k: bf16(g[k]) for k in ("x", "ctx", "ck", "cv", "y", "nk", "nv")}
    return g, wts, t, (dim, ffn, heads, f_cur, h, w)


def test_oracle_block_matches_reference_block(golden):
    """oracle.block (bf16 Linears) vs the reference WanAttentionBlock, streaming + cache."""
    from oracle import block as oblock
    g, wts, t, (dim, ffn, heads, f_cur, h, w) = _block_golden(golden)
    d = dim // heads
    tdim, hdim, wdim = onum.rope_axis_dims(d)
    freqs = torch.cat([onum.rope_params(1024, tdim), onum.rope_params(1024, hdim),
                       onum.rope_params(1024, wdim)], dim=1)
    y, nk, nv = oblock.block_forward(
        wts, t["x"][0], torch.from_numpy(g["e"])[0], t["ctx"][0], grid=(f_cur, h, w),
        freqs=freqs, t_offset=3, cache_k=t["ck"][0], cache_v=t["cv"][0], kv_len=9,
        block_hw=(2, 2), radius_hw=(1, 1), block_t=3, heads=heads, linear="bf16")
    ref = t["y"][0]
    assert onum.cosine(y.float(), ref.float()) > 0.99999
    assert (y.float() - ref.float()).abs().max() < 0.05
    assert torch.equal(nk, t["nk"][0]) and torch.equal(nv, t["nv"][0])


def test_oracle_model_matches_reference_wanmodel(golden):
    """oracle.model (embeddings, blocks with bf16 Linears, Head, unpatchify) vs two
    streaming chunks of the reference's own WanModel._forward_inference, the second
    over the first chunk's KV cache (tests/golden/gen_golden.py, gen_model)."""
    from types import SimpleNamespace

    from oracle import model as omodel
    g = golden("model")
    dim, ffn, heads, layers, c_in, c_out, text_dim, text_len, f, H, W = (int(v) for v in g["dims"])
    sd = {}
    for k, v in g.items():
        if k.startswith("w."):
            t = torch.from_numpy(v)
            sd[k[2:]] = t.view(torch.bfloat16) if t.dtype == torch.int16 else t
    cfg = SimpleNamespace(dim=dim, num_heads=heads, num_layers=layers, patch_size=(1, 2, 2),
                          freq_dim=256, text_len=text_len, eps=1e-6, rope_rows=1024,
                          block_hw=(2, 2), block_radius_hw=(1, 1), block_t=3, out_dim=c_out)
    ctx = bf16(g["ctx"])
    caches = None
    for i in range(2):
        out, caches = omodel.forward_chunk(sd, cfg, bf16(g[f"lat{i}"]), 625.0, ctx, caches=caches,
                                           t_offset=3 * i, kv_len=9, linear="bf16")
        ref = bf16(g[f"out{i}"])
        assert out.shape == ref.shape == (c_out, f, H, W)
        assert onum.cosine(out.float(), ref.float()) > 0.99999, i
        assert (out.float() - ref.float()).abs().max() < 0.05, i
    # the second layer's cache after the second chunk (roped K, raw V, 6 frames).
    # Layer 1's input already carries layer 0's bf16 rounding differences (the
    # reference's CPU attention and Linears accumulate in other orders), so about
    # 30% of its values sit an ulp or so away: compared by cosine, not bits
    nk, nv = caches[1]
    L = f * (H // 2) * (W // 2)
    assert nk.shape[0] == 2 * L
    for got, key in ((nk, "k1_layer1"), (nv, "v1_layer1")):
        ref = bf16(g[key]).reshape(got.shape)
        assert onum.cosine(got.float(), ref.float()) > 0.99999, key


UPSAMPLER_CASES = {
    "x2_replicate": dict(num_blocks=2, upsample_scale=2, residual=False,
                         memory_init="replicate"),
    "x4_residual": dict(num_blocks=1, upsample_scale=4, residual=True, residual_scale=0.5,
                        memory_init="zero"),
}


def upsampler_case(g, name):
    """(state dict, bf16 input, bf16 reference output, fp32 reference output) of a
    golden FlashLatentUpsampler case."""
    pre = name + ".sd."
    sd = {k[len(pre):]: torch.from_numpy(g[k]).view(torch.bfloat16) for k in g
          if k.startswith(pre)}
    return (sd, torch.from_numpy(g[name + ".x"]).view(torch.bfloat16),
            torch.from_numpy(g[name + ".y"]).view(torch.bfloat16),
            torch.from_numpy(g[name + ".y32"]))


@pytest.mark.parametrize("name", sorted(UPSAMPLER_CASES))
def test_oracle_upsampler_matches_reference(golden, name):
    """The oracle's latent upsampler against the reference FlashLatentUpsampler run
    in bf16 (the pipeline's precision) and in fp32: bf16-rounded at the same
    points, it sits about 10x closer to the bf16 run (only accumulation order
    differs; ~98% of the values bit-equal) than either does to fp32."""
    from oracle import upsampler as ou
    sd, x, y, y32 = upsampler_case(golden("upsampler"), name)
    out = ou.upsample(sd, x, **UPSAMPLER_CASES[name])
    assert out.shape == y.shape
    assert onum.rel_fro(out, y.double()) < 2e-3
    assert onum.rel_fro(out, y32.double()) < 1e-2
    assert float((out == y.double()).double().mean()) > 0.95


def test_oracle_vae_decode_matches_reference(golden):
    """The oracle's Wan2.2 VAE decode against the reference WanVAE_.decode:
    unrounded, it reproduces the fp32 run to float precision (the caches, the
    skipped first time_conv, DupUp3D, the phase of every upsample, attention and
    unpatchify all as the reference has them); with the bf16 rounding points it
    sits within the bf16 run's own distance from fp32 (about 1.3% at these
    random weights: ~30 convs amplify each rounding), cosine 0.9999."""
    from oracle import vae as ov
    from tests.golden_cases import vae_state_dict
    g = golden("vae")
    sd = vae_state_dict(g)
    z = torch.from_numpy(g["z"]).view(torch.bfloat16)
    mean, std = torch.from_numpy(g["mean"]), torch.from_numpy(g["std"])
    y = torch.from_numpy(g["y"]).view(torch.bfloat16).double()
    y32 = torch.from_numpy(g["y32"]).double()
    ye = ov.Decoder(sd, bf16=False).decode(z, mean, std)
    assert ye.shape == y32.shape == (3, 9, 64, 96)
    assert onum.rel_fro(ye, y32) < 1e-5
    yb = ov.Decoder(sd).decode(z, mean, std)
    assert onum.rel_fro(yb, y) < 2.5e-2 and onum.cosine(yb, y) > 0.9995
    assert onum.rel_fro(y, y32) > 0.5 * onum.rel_fro(yb, y)   # the same noise level
