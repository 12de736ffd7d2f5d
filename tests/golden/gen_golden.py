"""Generate the golden vectors in this directory by EXECUTING THE REFERENCE.

The reference (AMAP-ML/DreamX-Creator) ships no tests or fixtures for its
SR-DiT hot path, so its outputs are produced here, on the CPU, by importing its
own modules from a checkout of the repository:

    python tests/golden/gen_golden.py /path/to/DreamX-Creator

Everything is seeded. The fixtures pin the CPU oracle (``oracle/``), which in
turn checks the CUDA path; nothing at test or bench time reads the reference.

Files:
  plans.npz     params rows of ``blockgrid_triton.build_plan`` for the specs
                ``attention.mask_free_window_attention`` itself builds (recorded
                by swapping its ``_blockgrid_triton_attend`` for a recorder)
  winattn.npz   ``mask_free_window_attention(attn_impl="sdpa")`` outputs
  rope.npz      ``rope_apply`` outputs
  quant.npz     ``_quantize_rowwise_impl`` outputs
  norms.npz     ``WanLayerNorm`` / ``WanRMSNorm`` outputs
  block.npz     one ``WanAttentionBlock`` streaming forward (bf16, window attn)
  model.npz     two streaming chunks of a small ``WanModel`` (``_forward_inference``:
                patch / time / text embeddings, window-attention blocks, ``Head``,
                ``unpatchify``), the second over the first chunk's KV cache
  upsampler.npz ``FlashLatentUpsampler`` forwards (bf16 and fp32) of two small
                configurations: the shipped one's structure (x2, replicate
                memory, no residual) and a x4 two-stage head with the residual
                skip head and zero memory
  vae.npz       ``WanVAE_.decode`` (the Wan2.2 decoder at a small width) of a
                3-frame latent, bf16 and fp32

The only argument is the path of the reference checkout; nothing here assumes
where it lives.
"""
from __future__ import annotations

import pathlib
import sys
import warnings

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
warnings.filterwarnings("ignore")


def load_reference(root: str):
    sys.path.insert(0, str(pathlib.Path(root) / "video_refiner"))
    from wan.modules.sr_dit import attention, blockgrid_triton, fp8_linear, models
    return attention, blockgrid_triton, fp8_linear, models


def spec_fields(spec):
    return {k: (-1 if v is None else v) for k, v in spec._asdict().items()
            if k not in ("query_grain", "anchor_hw")}


# (name, f_cur, f_cache, h, w, block_t, block_hw, radius_hw, radius_t, anchor_mode,
#  anchor_hw, causal_chunk_frames, causal_kv_span)
PLAN_CASES = [
    ("cfg1_8x8_r0", 3, 0, 18, 32, 3, (8, 8), (0, 0), None, None, None, None, None),
    ("cfg1_4x4_r3", 3, 0, 18, 32, 3, (4, 4), (3, 3), None, None, None, None, None),
    ("2k_4x4_r3_f3", 3, 0, 36, 64, 3, (4, 4), (3, 3), None, None, None, None, None),
    ("2k_4x4_r3_f6", 3, 3, 36, 64, 3, (4, 4), (3, 3), None, None, None, None, None),
    ("2k_4x4_r3_f12", 3, 9, 36, 64, 3, (4, 4), (3, 3), None, None, None, None, None),
    ("2k_4x4_r3_f12_frame", 3, 9, 36, 64, 3, (4, 4), (3, 3), None, "frame", None, None, None),
    ("2k_4x4_r3_f6_chunk", 3, 3, 36, 64, 3, (4, 4), (3, 3), None, "chunk", None, None, None),
    ("2k_8x8_r0_f6", 3, 3, 36, 64, 3, (8, 8), (0, 0), None, None, None, None, None),
    ("2k_8x8_r0_f12_frame", 3, 9, 36, 64, 3, (8, 8), (0, 0), None, "frame", None, None, None),
    ("2k_4x4_r3_harvest", 1, 0, 36, 64, 3, (4, 4), (3, 3), None, None, None, None, None),
    ("odd_f5", 2, 3, 7, 10, 3, (3, 4), (1, 2), None, None, None, None, None),
    ("odd_frame", 2, 3, 7, 10, 3, (3, 4), (1, 2), None, "frame", None, None, None),
    ("native_anchor", 2, 2, 8, 12, 2, (4, 4), (1, 1), None, "frame", (4, 6), None, None),
    ("hist_rt1", 3, 6, 12, 16, 3, (4, 4), (1, 2), 1, None, None, None, None),
    ("parallel_causal", 6, 0, 8, 8, 3, (4, 4), (1, 1), None, None, None, 3, 6),
]


def gen_plans(attention, bgt):
    recorded = {}

    def recorder(spec, q_i, full_k, full_v, *, anchor_k=None, anchor_v=None,
                 anchor_align="frame", anchor_window_scope="window"):
        mode = None if anchor_k is None else ("frame" if anchor_align == "frame" else "chunk")
        recorded["spec"] = spec
        recorded["mode"] = mode
        return q_i.new_zeros(q_i.shape)

    orig = attention._blockgrid_triton_attend
    attention._blockgrid_triton_attend = recorder
    out = {}
    try:
        for (name, f_cur, f_cache, h, w, bt, bhw, rhw, rt, amode, ahw, ccf, cks) in PLAN_CASES:
            n, d = 1, 8
            L = h * w
            q = torch.zeros(1, f_cur * L, n, d)
            ck = torch.zeros(1, f_cache * L, n, d) if f_cache else None
            akw = {}
            if amode is not None:
                La = L if ahw is None else ahw[0] * ahw[1]
                akw = dict(anchor_k=torch.zeros(1, f_cur * La, n, d),
                           anchor_v=torch.zeros(1, f_cur * La, n, d),
                           anchor_align=amode, anchor_hw=ahw)
            attention.mask_free_window_attention(
                q, q, q, torch.tensor([[f_cur, h, w]]), pre_cache_k=ck, pre_cache_v=ck,
                kv_len=9, attn_impl="triton", block_t=bt, block_hw=bhw,
                block_radius_hw=rhw, block_radius_t=rt, causal_chunk_frames=ccf,
                causal_kv_span=cks, **akw)
            spec, mode = recorded["spec"], recorded["mode"]
            plan = bgt.build_plan(spec, anchor_mode=mode)
            out[f"{name}.params"] = plan["params"].numpy()
            meta = [plan["n_w"], plan["block_m"], plan["m_tiles"], plan["block_n"],
                    plan["hr_base"], plan["p_stride"]]
            out[f"{name}.meta"] = np.asarray(meta, dtype=np.int64)
            sf = spec_fields(spec)
            out[f"{name}.spec"] = np.asarray(
                [sf[k] for k in ("f_cur", "f_kv", "h", "w", "block_t", "bh", "bw", "rh", "rw",
                                 "hist", "rt", "chunk_frames", "streaming")], dtype=np.int64)
            ahw_s = spec.anchor_hw
            out[f"{name}.anchor_hw"] = np.asarray(ahw_s if ahw_s is not None else (-1, -1))
            out[f"{name}.mode"] = np.asarray({None: 0, "chunk": 1, "frame": 2}[mode])
    finally:
        attention._blockgrid_triton_attend = orig
    np.savez_compressed(HERE / "plans.npz", **out)
    print("plans:", len(PLAN_CASES))


def rope_freqs(models, head_dim=128, max_len=1024):
    t, h, w = models._rope_axis_dims(head_dim)
    return torch.cat([models.rope_params(max_len, t), models.rope_params(max_len, h),
                      models.rope_params(max_len, w)], dim=1)


def gen_winattn(attention, models):
    out = {}
    freqs = rope_freqs(models)
    # config 1 (BASELINE): seed 0, q,k,v ~ N(0,1) fp32 [1,1728,24,128] in that order,
    # grid (3,18,32), RoPE theta 1e4, reference PyTorch (non-Triton) path.
    torch.manual_seed(0)
    q = torch.randn(1, 1728, 24, 128)
    k = torch.randn(1, 1728, 24, 128)
    v = torch.randn(1, 1728, 24, 128)
    grid = torch.tensor([[3, 18, 32]])
    qr = models.rope_apply(q, grid, freqs)
    kr = models.rope_apply(k, grid, freqs)
    for tag, bhw, rhw in (("cfg1_8x8_r0", (8, 8), (0, 0)), ("cfg1_4x4_r3", (4, 4), (3, 3))):
        o, _, _ = attention.mask_free_window_attention(
            qr, kr, v, grid, attn_impl="sdpa", block_t=3, block_hw=bhw, block_radius_hw=rhw)
        o = o[0]
        out[f"{tag}.out_h0"] = o[:, 0].numpy().astype(np.float32)
        out[f"{tag}.sum"] = np.asarray([float(o.double().sum()), float(o.double().abs().sum()),
                                        float((o.double() ** 2).sum())])
        out[f"{tag}.rows"] = o[::97].numpy().astype(np.float32)
    # streaming with a cache and an LQ anchor on a small grid, 2 heads
    g = torch.Generator().manual_seed(1)
    f_cur, f_cache, h, w, n, d = 3, 3, 8, 12, 2, 128
    L = h * w
    q = torch.randn(1, f_cur * L, n, d, generator=g)
    k = torch.randn(1, f_cur * L, n, d, generator=g)
    v = torch.randn(1, f_cur * L, n, d, generator=g)
    ck = torch.randn(1, f_cache * L, n, d, generator=g)
    cv = torch.randn(1, f_cache * L, n, d, generator=g)
    ak = torch.randn(1, f_cur * L, n, d, generator=g)
    av = torch.randn(1, f_cur * L, n, d, generator=g)
    # inputs are regenerated by the tests from the same seeded generator; the
    # checksums below catch a generator that does not reproduce them
    out["stream.input_sums"] = np.asarray([float(t.double().sum()) for t in (q, k, v, ck, cv, ak, av)])
    gr = torch.tensor([[f_cur, h, w]])
    for tag, akw in (("none", {}), ("frame", dict(anchor_k=ak, anchor_v=av, anchor_align="frame")),
                     ("chunk", dict(anchor_k=ak, anchor_v=av, anchor_align="chunk"))):
        o, nck, ncv = attention.mask_free_window_attention(
            q, k, v, gr, pre_cache_k=ck, pre_cache_v=cv, kv_len=4, attn_impl="sdpa",
            block_t=3, block_hw=(4, 4), block_radius_hw=(1, 1), **akw)
        out[f"stream.{tag}.out"] = o[0].numpy()
        if tag == "none":
            out["stream.cache_k"] = nck[0].numpy()
    np.savez_compressed(HERE / "winattn.npz", **out)
    print("winattn ok")


def gen_rope(models):
    g = torch.Generator().manual_seed(2)
    freqs = rope_freqs(models)
    grid = torch.tensor([[2, 5, 7]])
    x = torch.randn(1, 70, 2, 128, generator=g).to(torch.bfloat16)
    y = models.rope_apply(x, grid, freqs, t_offset=3)
    xf = torch.randn(1, 70, 2, 128, generator=g)
    yf = models.rope_apply(xf, grid, freqs, t_offset=0)
    np.savez_compressed(HERE / "rope.npz", x=x[0].view(torch.int16).numpy(),
                        y=y[0].view(torch.int16).numpy(), xf=xf[0].numpy(), yf=yf[0].numpy(),
                        freqs_re=freqs.real.numpy()[:16], freqs_im=freqs.imag.numpy()[:16])
    print("rope ok")


def gen_quant(fp8):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 512, generator=g)
    mask = torch.rand(64, 512, generator=g) < 0.001
    x = torch.where(mask, x * 20, x).to(torch.bfloat16)
    x[5] = 0
    q, s = fp8._quantize_rowwise_impl(x)
    np.savez_compressed(HERE / "quant.npz", x=x.view(torch.int16).numpy(),
                        q=q.view(torch.uint8).numpy(), s=s.numpy())
    print("quant ok")


def gen_norms(models):
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(32, 256, generator=g) * 3 + 0.5).to(torch.bfloat16)
    ln = models.WanLayerNorm(256, 1e-6)
    lna = models.WanLayerNorm(256, 1e-6, elementwise_affine=True)
    with torch.no_grad():
        lna.weight.copy_(torch.randn(256, generator=g))
        lna.bias.copy_(torch.randn(256, generator=g))
    lna = lna.to(torch.bfloat16)
    rms = models.WanRMSNorm(256, eps=1e-6)
    with torch.no_grad():
        rms.weight.copy_(torch.randn(256, generator=g))
    rms = rms.to(torch.bfloat16)
    with torch.no_grad():
        y_ln, y_lna, y_rms = ln(x), lna(x), rms(x)
    np.savez_compressed(HERE / "norms.npz", x=x.view(torch.int16).numpy(),
                        ln=y_ln.view(torch.int16).numpy(), lna=y_lna.view(torch.int16).numpy(),
                        lna_w=lna.weight.view(torch.int16).numpy(),
                        lna_b=lna.bias.view(torch.int16).numpy(),
                        rms=y_rms.view(torch.int16).numpy(),
                        rms_w=rms.weight.view(torch.int16).numpy())
    print("norms ok")


def gen_block(models):
    dim, ffn, heads, f_cur, h, w, ctx_len = 256, 512, 2, 3, 4, 6, 16
    torch.manual_seed(5)
    blk = models.WanAttentionBlock("t2v_cross_attn", dim, ffn, heads, (-1, -1), True, True, 1e-6,
                                   stream_chunk_size=3)
    g = torch.Generator().manual_seed(6)
    with torch.no_grad():
        for name, p in sorted(blk.named_parameters()):
            if name.endswith("bias"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.01)
            elif "norm" in name:
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
            elif name == "modulation":
                p.copy_(torch.randn(p.shape, generator=g) / dim ** 0.5)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    blk = blk.to(torch.bfloat16)
    blk.modulation.data = blk.modulation.data.float()
    attn = blk.self_attn
    attn.use_window_attn = True
    attn.window_attn_impl = "sdpa"
    attn.window_block_hw = (2, 2)
    attn.window_block_radius_hw = (1, 1)
    L = h * w
    x = torch.randn(1, f_cur * L, dim, generator=g).to(torch.bfloat16)
    e = torch.randn(1, 6, dim, generator=g).float() * 0.1
    ctx = torch.randn(1, ctx_len, dim, generator=g).to(torch.bfloat16)
    ck = torch.randn(1, 3 * L, heads, dim // heads, generator=g).to(torch.bfloat16)
    cv = torch.randn(1, 3 * L, heads, dim // heads, generator=g).to(torch.bfloat16)
    t, hd, wd = models._rope_axis_dims(dim // heads)
    freqs = torch.cat([models.rope_params(1024, t), models.rope_params(1024, hd),
                       models.rope_params(1024, wd)], dim=1)
    grid = torch.tensor([[f_cur, h, w]])
    with torch.no_grad():
        y, nk, nv = blk(x, e=e, seq_lens=torch.tensor([f_cur * L]), grid_sizes=grid, freqs=freqs,
                        context=ctx, context_lens=None, temporal_offset=3, is_stream=True,
                        pre_cache_k=ck, pre_cache_v=cv, kv_len=9)
    def bits(t):  # bf16 tensors stored as their 16-bit patterns
        return t.contiguous().view(torch.int16).numpy()
    sd = {f"w.{k}": (bits(v) if v.dtype == torch.bfloat16 else v.numpy())
          for k, v in blk.state_dict().items()}
    np.savez_compressed(HERE / "block.npz", x=bits(x), e=e.numpy(), ctx=bits(ctx), ck=bits(ck),
                        cv=bits(cv), y=bits(y), nk=bits(nk), nv=bits(nv),
                        dims=np.asarray([dim, ffn, heads, f_cur, h, w, ctx_len, 3]), **sd)
    print("block ok")


def gen_model(models):
    """A small WanModel (2 blocks, dim 128, 2 heads of 64, window attention 2x2
    radius 1 on the sdpa backend), seeded weights; two 3-frame chunks through its
    streaming ``forward`` -> ``_forward_inference`` (models.py:1877-2002), the second
    at temporal offset 3 over the first chunk's returned KV cache. The time
    embedding, time projection and head are kept in fp32 (what the CUDA fp32
    autocast around them gives on the GPU; the CPU autocast is a no-op), the rest
    in bf16."""
    dim, ffn, heads, layers, c_in, c_out, text_dim, text_len = 128, 256, 2, 2, 16, 16, 32, 8
    f, H, W = 3, 8, 12
    torch.manual_seed(7)
    m = models.WanModel(model_type="t2v", patch_size=(1, 2, 2), text_len=text_len, in_dim=c_in,
                        dim=dim, ffn_dim=ffn, freq_dim=256, text_dim=text_dim, out_dim=c_out,
                        num_heads=heads, num_layers=layers, qk_norm=True, cross_attn_norm=True,
                        eps=1e-6, stream_chunk_size=3)
    m.enable_window_attention(window_block_hw=(2, 2), window_block_radius_hw=(1, 1),
                              window_attn_impl="sdpa")
    g = torch.Generator().manual_seed(8)
    with torch.no_grad():
        for name, p in sorted(m.named_parameters()):
            if name.endswith("modulation"):
                p.copy_(torch.randn(p.shape, generator=g) / dim ** 0.5)
            elif name.endswith("bias"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.01)
            elif "norm" in name:
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    m = m.to(torch.bfloat16)
    for sub in (m.time_embedding, m.time_projection, m.head):
        sub.float()
    for blk in m.blocks:
        blk.modulation.data = blk.modulation.data.float()
    m.eval()
    lat = [torch.randn(c_in, f, H, W, generator=g).to(torch.bfloat16) for _ in range(2)]
    ctx = torch.randn(text_len - 2, text_dim, generator=g).to(torch.bfloat16)  # padded by the model
    L = f * (H // 2) * (W // 2)
    outs, caches = [], None
    with torch.no_grad():
        for i, x in enumerate(lat):
            o, caches = m(x=[x], t=torch.tensor([625.0]), context=[ctx], seq_len=L,
                          temporal_offset=3 * i, kv_caches=caches, kv_len=9, is_stream=True)
            outs.append(o[0])

    def bits(t):
        return t.contiguous().view(torch.int16).numpy()
    sd = {f"w.{k}": (bits(v) if v.dtype == torch.bfloat16 else v.numpy())
          for k, v in m.state_dict().items()}
    np.savez_compressed(HERE / "model.npz", lat0=bits(lat[0]), lat1=bits(lat[1]), ctx=bits(ctx),
                        out0=bits(outs[0]), out1=bits(outs[1]),
                        k1_layer1=bits(caches[1][0][0]), v1_layer1=bits(caches[1][1][0]),
                        dims=np.asarray([dim, ffn, heads, layers, c_in, c_out, text_dim,
                                         text_len, f, H, W]), **sd)
    print("model ok")


# (name, constructor arguments, (B, T, H, W))
UPSAMPLER_CASES = [
    ("x2_replicate", dict(in_channels=16, out_channels=16, mid_channels=64, num_blocks=2,
                          upsample_scale=2, residual=False, memory_init="replicate"),
     (2, 3, 6, 10)),
    ("x4_residual", dict(in_channels=16, out_channels=16, mid_channels=64, num_blocks=1,
                         upsample_scale=4, residual=True, residual_scale=0.5,
                         memory_init="zero"),
     (1, 2, 5, 6)),
]


def gen_upsampler(root: str):
    import importlib.util
    path = (pathlib.Path(root) / "video_refiner" / "wan" / "modules" / "latent_upsampler"
            / "flash_latent_up.py")
    spec = importlib.util.spec_from_file_location("flash_latent_up", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = {}
    for i, (name, kw, (B, T, H, W)) in enumerate(UPSAMPLER_CASES):
        torch.manual_seed(100 + i)
        # PyTorch's default conv init (random weights), the final projection kept
        m = mod.FlashLatentUpsampler(**kw, init_mode="default", zero_init_final=False).eval()
        m = m.to(torch.bfloat16)
        x = torch.randn(B, kw["in_channels"], T, H, W).to(torch.bfloat16)
        with torch.no_grad():
            y = m(x)
            y32 = m.float()(x.float())
        for k, v in m.state_dict().items():
            out[f"{name}.sd.{k}"] = v.to(torch.bfloat16).view(torch.int16).numpy()
        out[f"{name}.x"] = x.view(torch.int16).numpy()
        out[f"{name}.y"] = y.view(torch.int16).numpy()
        out[f"{name}.y32"] = y32.numpy()
    np.savez_compressed(HERE / "upsampler.npz", **out)
    print("upsampler ok")


def gen_vae(root: str):
    """WanVAE_.decode (the Wan2.2 decoder: dim_mult [1, 2, 4, 4], 2 residual
    blocks, temporal upsampling [True, True, False]) at a small width (dec_dim
    64) on a 48-channel latent of 3 frames x 4 x 6, in bf16 (the pipeline's
    precision) and fp32. Seeded random weights (every decoder parameter, the RMS_norm
    gammas and the attention projection included), regenerated by the tests from
    the stored parameter names and shapes (``tests.golden_cases.vae_param``)."""
    import importlib.util
    path = pathlib.Path(root) / "video_refiner" / "wan" / "modules" / "vae2_2.py"
    spec = importlib.util.spec_from_file_location("vae2_2", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.path.insert(0, str(HERE.parents[1]))
    from tests.golden_cases import vae_param
    m = mod.WanVAE_(dim=32, dec_dim=64, z_dim=48, dim_mult=[1, 2, 4, 4], num_res_blocks=2,
                    attn_scales=[], temperal_downsample=[False, True, True]).eval()
    names = sorted(n for n, _ in m.named_parameters()
                   if n.startswith("decoder.") or n.startswith("conv2."))
    prms = dict(m.named_parameters())
    with torch.no_grad():
        for i, n in enumerate(names):
            prms[n].copy_(vae_param(n, tuple(prms[n].shape), i))
    z = torch.randn(1, 48, 3, 4, 6)
    g = torch.Generator().manual_seed(3)
    mean = 0.2 * torch.randn(48, generator=g)
    std = 0.5 + torch.rand(48, generator=g)
    out = {}
    with torch.no_grad():
        mb = m.to(torch.bfloat16)
        zb = z.to(torch.bfloat16)
        y = mb.decode(zb, [mean.to(torch.bfloat16), 1.0 / std.to(torch.bfloat16)])
        m32 = mb.float()
        y32 = m32.decode(zb.float(), [mean, 1.0 / std])
    out["param_names"] = np.asarray(names)
    shapes = [tuple(prms[n].shape) for n in names]
    out["param_ndims"] = np.asarray([len(sh) for sh in shapes])
    out["param_shapes"] = np.asarray([list(sh) + [0] * (5 - len(sh)) for sh in shapes])
    out["z"] = zb[0].view(torch.int16).numpy()
    out["mean"] = mean.numpy()
    out["std"] = std.numpy()
    out["y"] = y[0].view(torch.int16).numpy()
    out["y32"] = y32[0].numpy()
    np.savez_compressed(HERE / "vae.npz", **out)
    print("vae ok", tuple(y.shape))


GENERATORS = ("plans", "quant", "norms", "rope", "winattn", "block", "model", "upsampler", "vae")


def main():
    if len(sys.argv) < 2 or any(a not in GENERATORS for a in sys.argv[2:]):
        raise SystemExit("usage: python tests/golden/gen_golden.py <path of the reference "
                         "checkout> [" + " | ".join(GENERATORS) + " ...] (writes the .npz "
                         "files beside this script; all of them by default)")
    which = set(sys.argv[2:]) or set(GENERATORS)
    torch.set_num_threads(8)
    if which - {"upsampler", "vae"}:
        attention, bgt, fp8, models = load_reference(sys.argv[1])
    if "plans" in which:
        gen_plans(attention, bgt)
    if "quant" in which:
        gen_quant(fp8)
    if "norms" in which:
        gen_norms(models)
    if "rope" in which:
        gen_rope(models)
    if "winattn" in which:
        gen_winattn(attention, models)
    if "block" in which:
        gen_block(models)
    if "model" in which:
        gen_model(models)
    if "upsampler" in which:
        gen_upsampler(sys.argv[1])
    if "vae" in which:
        gen_vae(sys.argv[1])


if __name__ == "__main__":
    main()
