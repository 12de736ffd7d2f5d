#!/usr/bin/env python
"""SR-DiT 5B 2K refinement throughput on B200 (latent-frames/s).

One step = one autoregressive refinement chunk of BASELINE config 3: 3 latent
frames at 2048x1152 (latent 48x3x72x128 -> 36x64 tokens/frame, 6912 tokens),
a 3-frame KV-cache prefix (the denoise forward attends f_kv = 6 frames), a
512-token N(0,1) 4096-d text context, 3x8x8 block-grid windows, fp8 Linears.
The step is the reference pipeline's per-chunk work
(pipeline_sr/causal_inference.py:858-976): a denoise forward at t=625, the
flow->x0 update, and the KV-refresh forward at t=0 -- 2 x 30 blocks. The ring is
restored to the 3-frame prefix before every step, so every step does the same
work. Weights are seeded random (no checkpoint); inputs are seeded synthetic.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

N > 1 (under torchrun): tensor parallelism over N ranks on one clip (heads and
FFN sharded, sequence-parallel residual stream; strong scaling), with
--parallel spatial a strip of token columns per rank (strong scaling), or with
--parallel replicas every rank refines its own clip (weak scaling); the step
time is the max over ranks.

Other lines: --clip (config 5: a 121-frame clip over the rolling cache; with
--pipeline the whole latent path -- upsampler, refiner loop, VAE decode);
--micro (one kernel, or the latent upsampler / the VAE decode, in isolation,
beside the reference's own GPU ops where they exist).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "2K SR-DiT refine latent-frames/s @1/2/4/8 B200; fp8 GEMM & win-attn % of roofline"
UNIT = "latent-frames/s"
FRAMES_PER_STEP = 3
# DRAM bytes (read + write) per srdit_fp8_gemm launch, averaged over the six
# GEMM launches of one block: ncu dram__bytes_read.sum + dram__bytes_write.sum
# of one launch of each of the step's four shapes (6912 x {9216, 3072, 14336} x
# 3072 and 6912 x 3072 x 14336), weighted 1 / 3 / 1 / 1 per block.
GEMM_TRAFFIC_PER_LAUNCH = 142.0e6
LAT_SHAPE = (48, 3, 72, 128)
CTX_SHAPE = (512, 4096)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--geometry", default="8x8r0", choices=["8x8r0", "4x4r3"])
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--tp-comm", default="fused", choices=["fused", "nccl"],
                    help="TP collectives fused into the kernels over peer memory, or NCCL")
    ap.add_argument("--parallel", default="tp", choices=["tp", "spatial", "replicas"],
                    help="N > 1: tensor parallelism over one clip (strong scaling, the "
                         "reference's DTensor-style TP), the spatial partition of one clip "
                         "(each GPU refines a strip of token columns with the full model; "
                         "a K/V halo for windows of radius > 0), or one clip per GPU (weak "
                         "scaling)")
    ap.add_argument("--halo", default="peer", choices=["peer", "collective"],
                    help="--parallel spatial with windows of radius > 0 along w: the K/V "
                         "halo columns stored into the neighbours' rings by the ring-write "
                         "kernel over NVLink, or sent with NCCL point-to-point calls")
    ap.add_argument("--anchor", default="none", choices=["none", "serial", "overlap"],
                    help="LQ-anchor steps (the shipped default denoise): every step also "
                         "harvests an anchor from a 3-frame LR chunk and denoises frame-"
                         "aligned to it; 'serial' harvests inside the step, 'overlap' "
                         "harvests the next step's anchor on a side stream")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graphs", action="store_true",
                    help="issue every kernel from Python instead of replaying the step's "
                         "CUDA graph")
    ap.add_argument("--micro", default=None,
                    choices=["gemm", "attn", "quant", "ln", "rope", "conv", "upsampler",
                             "conv3d", "vae"],
                    help="time one kernel (or the latent upsampler) in isolation instead of "
                         "the model step")
    ap.add_argument("--shape", default=None,
                    help="micro shape: gemm M,N,K | attn f_kv | quant/ln/rope M,K | "
                         "conv F,H,W,cin,n_src,cout | upsampler T,H,W (LR latent) | "
                         "conv3d F,H,W,cin,cout,kt,kh | vae T,h,w (latent)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--epi", default="store", choices=["store", "gelu", "gated_res", "res"],
                    help="micro gemm: the epilogue")
    ap.add_argument("--pipeline", action="store_true",
                    help="with --clip at N = 1: the whole latent path of a clip -- the "
                         "latent upsampler on the LR latent, the noise mix, the refiner "
                         "loop, and the Wan2.2 VAE decode to pixels -- timed stage by stage")
    ap.add_argument("--clip", action="store_true",
                    help="BASELINE config 5: a 121-frame clip (33 latent frames, 11 chunks) "
                         "over the rolling KV cache; sustained latent-frames/s and per-chunk "
                         "p50 / p99 latency")
    return ap.parse_args()


def run_micro(args):
    """One kernel in isolation: median CUDA-event time over --iters launches, the L2
    cleaned between launches by reading a 512 MB buffer (no dirty lines left)."""
    srdit = importlib.import_module("dreamx-creator_b200")
    ops = srdit.ops
    dev = torch.device("cuda", 0)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)

    def timeit(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(args.iters):
            flush.max()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    peaks, kind = load_peaks()
    res = {"micro": args.micro}
    if args.micro == "gemm":
        M, N, K = (int(v) for v in (args.shape or "6912,14336,3072").split(","))
        a = torch.randn(M, K, device=dev, generator=g).to(torch.float8_e4m3fn)
        w = torch.randn(N, K, device=dev, generator=g).to(torch.float8_e4m3fn)
        sa, sb = torch.rand(M, device=dev), torch.rand(N, device=dev)
        bias = torch.randn(N, device=dev).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        extra = {}
        if args.epi == "gelu":
            extra = dict(epilogue="gelu", row_amax=torch.zeros(M, device=dev))
        elif args.epi in ("gated_res", "res"):
            extra = dict(epilogue=args.epi, residual=torch.randn(M, N, device=dev).to(torch.bfloat16))
            if args.epi == "gated_res":
                extra["gate"] = torch.randn(N, device=dev)
        ms = timeit(lambda: ops.fp8_gemm(a, sa, w, sb, bias, out, **extra))
        ref = timeit(lambda: torch._scaled_mm(a, w.t(), scale_a=sa.view(-1, 1),
                                              scale_b=sb.view(1, -1), bias=bias,
                                              out_dtype=torch.bfloat16))
        fl = 2 * M * N * K
        res.update(shape=[M, N, K], epilogue=args.epi, ms=ms, tflops=fl / ms / 1e9, cublaslt_ms=ref,
                   cublaslt_tflops=fl / ref / 1e9,
                   frac_of_2x_bf16_burst=fl / ms / 1e9 / (2 * peaks["bf16_tflops"]))
    elif args.micro == "attn":
        fkv = int(args.shape or 6)
        bhw, rhw = geometry(args.geometry)
        spec = srdit.blockgrid.make_spec(f_cur=3, f_kv=fkv, h=36, w=64, block_t=3, block_hw=bhw,
                                         block_radius_hw=rhw, streaming=True)
        plan = srdit.attention.cached_plan(spec)
        q = torch.randn(6912, 24, 128, device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn(fkv * 2304, 24, 128, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(fkv * 2304, 24, 128, device=dev, generator=g).to(torch.bfloat16)
        o = torch.empty_like(q)
        ms = timeit(lambda: srdit.attention.run_blockgrid_b200(q, k, v, o, plan=plan, f_cur=3,
                                                               h=36, w=64, n=24, d=128))
        fl = srdit.blockgrid.visible_flops(plan["params"], plan["p_stride"], 24, 128)
        res.update(geometry=args.geometry, f_kv=fkv, ms=ms, gflop=fl / 1e9,
                   tflops=fl / ms / 1e9, frac_of_bf16_burst=fl / ms / 1e9 / peaks["bf16_tflops"])
        ref = reference_winattn(args, srdit, dev, timeit, fkv, bhw, rhw, fl, peaks)
        if ref is not None:
            res["reference_triton"] = ref
    elif args.micro == "conv":
        F, H, W, cin, n_src, cout = (int(v) for v in (args.shape or "33,72,128,128,2,128")
                                     .split(","))
        x = torch.randn(F, H, W, cin, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(cout, n_src * cin, 3, 3, device=dev, generator=g) * 0.02)
        w = w.to(torch.bfloat16)
        b = torch.randn(cout, device=dev, generator=g).to(torch.bfloat16)
        w2, b2 = ops.conv_weight(w, n_src=n_src), ops.conv_bias(b)
        out = torch.empty(F, H, W, cout, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda: ops.conv3x3(x, w2, b2, frames_per_clip=F, n_src=n_src, relu=True,
                                        out=out))
        # cuDNN: the reference's bf16 nn.Conv2d on NCHW frames (the cat of the
        # block's two sources made once, outside the timing)
        xn = x.permute(0, 3, 1, 2).contiguous()
        if n_src == 2:
            xn = torch.cat([xn, torch.cat([xn[:1], xn[:-1]])], 1)
        ref = timeit(lambda: torch.relu(torch.nn.functional.conv2d(xn, w, b, padding=1)))
        fl = 2 * F * H * W * cout * 9 * cin * n_src
        res.update(shape=[F, H, W, cin, n_src, cout], ms=ms, tflops=fl / ms / 1e9,
                   cudnn_ms=ref, cudnn_tflops=fl / ref / 1e9,
                   frac_of_bf16_burst=fl / ms / 1e9 / peaks["bf16_tflops"])
    elif args.micro == "upsampler":
        res.update(run_upsampler_micro(args, dev, timeit, peaks))
    elif args.micro == "conv3d":
        F, H, W, cin, cout, kt, kh = (int(v) for v in (args.shape or "2,144,256,1024,1024,3,3")
                                      .split(","))
        x = torch.randn(F + kt - 1, H, W, cin, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(cout, cin, kt, kh, kh, device=dev, generator=g) * 0.01).to(torch.bfloat16)
        b = torch.randn(cout, device=dev, generator=g)
        w2 = ops.conv3d_weight(w)
        out = torch.empty(F, H, W, cout, device=dev, dtype=torch.bfloat16)
        ms = timeit(lambda: ops.conv3d(x, w2, b, kt=kt, kh=kh, out=out))
        # cuDNN: the reference's CausalConv3d on NCDHW (cache frames and the zero
        # spatial padding concatenated / padded once, outside the timing)
        xn = torch.nn.functional.pad(x.permute(3, 0, 1, 2)[None], (kh // 2,) * 4)
        bb = b.to(torch.bfloat16)
        ref = timeit(lambda: torch.nn.functional.conv3d(xn, w, bb))
        fl = 2 * F * H * W * cout * cin * kt * kh * kh
        res.update(shape=[F, H, W, cin, cout, kt, kh], ms=ms, tflops=fl / ms / 1e9,
                   cudnn_ms=ref, cudnn_tflops=fl / ref / 1e9,
                   frac_of_bf16_burst=fl / ms / 1e9 / peaks["bf16_tflops"])
    elif args.micro == "vae":
        res.update(run_vae_micro(args, dev, peaks))
    else:
        M, K = (int(v) for v in (args.shape or "6912,3072").split(","))
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        if args.micro == "quant":
            # the FFN's wide activation arrives with its row amax (GEMM epilogue)
            amax = x.float().abs().amax(-1) if K > 4096 else None
            ms = timeit(lambda: ops.quant_rowwise(x, amax=amax))
            byts = M * K * 2 + M * K + 4 * M
        elif args.micro == "ln":
            sh, sc = torch.randn(K, device=dev), torch.randn(K, device=dev)
            ms = timeit(lambda: ops.ln_mod_quant(x, 1e-6, shift=sh, scale=sc))
            byts = M * K * 2 + M * K + 4 * M
        else:
            mm = importlib.import_module("dreamx-creator_b200.model")
            cos, sin = mm.rope_tables(128, 1024, 1e4, dev)
            wt = torch.ones(K, device=dev, dtype=torch.bfloat16)
            dst = torch.empty_like(x)
            ms = timeit(lambda: ops.rms_rope(x, wt, 1e-6, dst, frame_tokens=2304, cos=cos, sin=sin,
                                             grid_h=36, grid_w=64))
            byts = 2 * M * K * 2
        res.update(shape=[M, K], ms=ms, gbs=byts / ms / 1e6,
                   frac_of_hbm=byts / ms / 1e6 / peaks["hbm_gbs"])
    res["peaks"] = kind
    print(json.dumps(res), flush=True)


REF_INSTALL = ROOT / "baseline" / "_ref"


def reference_attention():
    """The reference's attention module and Triton launcher module, imported from
    its install under baseline/_ref; None when it is not installed."""
    if not (REF_INSTALL / "wan" / "modules" / "sr_dit" / "attention.py").exists():
        return None
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    from wan.modules.sr_dit import attention as ref_attn
    from wan.modules.sr_dit import blockgrid_triton as ref_bgt
    return ref_attn, ref_bgt


def reference_winattn(args, srdit, dev, timeit, fkv, bhw, rhw, flops, peaks):
    """The reference's own GPU window attention on the same 2K chunk, on this GPU.

    - kernel: its Triton launcher (run_blockgrid_triton, blockgrid_triton.py:392-422)
      on the arguments its op passes it (its own plan, the cat([cache, chunk])
      K/V), and srdit_winattn_fwd (run_blockgrid_b200) on the same arguments;
    - op: the whole public op, mask_free_window_attention(attn_impl="triton")
      (attention.py:1376-1648), with its stock launcher and with the B200
      launcher installed at its seam (attention.install).
    Both outputs are compared element by element."""
    mods = reference_attention()
    if mods is None:
        return None
    ref_attn, _ = mods
    g = torch.Generator(device=dev).manual_seed(1)
    L, f_cur, f_cache = 36 * 64, 3, fkv - 3

    def rnd(frames):
        return torch.randn(1, frames * L, 24, 128, device=dev, generator=g).to(torch.bfloat16)

    q, k, v = rnd(f_cur), rnd(f_cur), rnd(f_cur)
    ck, cv = (rnd(f_cache), rnd(f_cache)) if f_cache else (None, None)
    grid = torch.tensor([[f_cur, 36, 64]])

    def op():
        return ref_attn.mask_free_window_attention(
            q, k, v, grid, pre_cache_k=ck, pre_cache_v=cv, kv_len=f_cache,
            attn_impl="triton", block_t=3, block_hw=bhw, block_radius_hw=rhw)[0]

    stock = ref_attn._run_blockgrid_triton
    seen = {}

    def recorder(*a, **kw):
        seen["a"], seen["kw"] = a, kw
        return stock(*a, **kw)

    ref_attn._run_blockgrid_triton = recorder
    try:
        op()
    finally:
        ref_attn._run_blockgrid_triton = stock
    (qf, kext, vext, out_t), kw = seen["a"], seen["kw"]
    out_b = torch.empty_like(out_t)
    t_ref = timeit(lambda: stock(qf, kext, vext, out_t, **kw))
    t_b = timeit(lambda: srdit.attention.run_blockgrid_b200(qf, kext, vext, out_b, **kw))
    torch.cuda.synchronize()
    diff = (out_b.float() - out_t.float()).abs()
    rel = (diff.norm() / out_t.float().norm()).item()
    t_op_ref = timeit(op)
    o_ref = op()
    srdit.attention.install(ref_attn)
    try:
        t_op_b = timeit(op)
        o_b = op()
    finally:
        ref_attn._run_blockgrid_triton = stock

    def dropin():
        return srdit.attention.mask_free_window_attention(
            q, k, v, grid, pre_cache_k=ck, pre_cache_v=cv, kv_len=f_cache, attn_impl="b200",
            block_t=3, block_hw=bhw, block_radius_hw=rhw)[0]

    t_dropin = timeit(dropin)
    o_d = dropin()
    torch.cuda.synchronize()
    return {
        "source": "reference installed under baseline/_ref (blockgrid_triton.py, attention.py)",
        "kernel_ms": t_ref, "kernel_tflops": flops / t_ref / 1e9,
        "kernel_frac_of_bf16_burst": flops / t_ref / 1e9 / peaks["bf16_tflops"],
        "b200_kernel_ms_same_args": t_b, "kernel_speedup": t_ref / t_b,
        "max_abs_diff": diff.max().item(), "rel_fro_diff": rel,
        "op_ms_triton": t_op_ref, "op_ms_b200": t_op_b, "op_speedup": t_op_ref / t_op_b,
        "op_max_abs_diff": (o_b.float() - o_ref.float()).abs().max().item(),
        # this repository's drop-in op (cache and chunk as two K/V segments, no cat)
        "dropin_op_ms": t_dropin, "dropin_op_speedup": t_op_ref / t_dropin,
        "dropin_max_abs_diff": (o_d.float() - o_ref.float()).abs().max().item(),
    }


def cudnn_upsampler(sd, x, *, num_blocks, scale):
    """The reference FlashLatentUpsampler's parallel forward (flash_latent_up.py:
    453-495; replicate memory, no residual) as its bf16 torch ops: cuDNN convs on
    NCHW frames, PixelShuffle, ReLU, the cat with the previous frames -- the
    reference's own execution path, for timing beside the B200 kernels."""
    B, C, T, H, W = x.shape
    h = x.permute(0, 2, 1, 3, 4).reshape(B * T, C, H, W)
    h = torch.nn.functional.conv2d(h, sd["pre_shuffle.0.weight"], sd["pre_shuffle.0.bias"],
                                   padding=1)
    h = torch.relu(torch.nn.functional.pixel_shuffle(h, scale))
    for i in range(num_blocks):
        hb = h.reshape(B, T, *h.shape[1:])
        past = torch.cat([hb[:, :1], hb[:, :-1]], 1).reshape(h.shape)
        p = f"blocks.{i}.conv"
        t = torch.relu(torch.nn.functional.conv2d(torch.cat([h, past], 1), sd[p + ".0.weight"],
                                                  sd[p + ".0.bias"], padding=1))
        t = torch.relu(torch.nn.functional.conv2d(t, sd[p + ".2.weight"], sd[p + ".2.bias"],
                                                  padding=1))
        t = torch.nn.functional.conv2d(t, sd[p + ".4.weight"], sd[p + ".4.bias"], padding=1)
        h = torch.relu(t + h)
    h = torch.nn.functional.conv2d(h, sd["final.weight"], sd["final.bias"], padding=1)
    return h.reshape(B, T, *h.shape[1:]).permute(0, 2, 1, 3, 4)


def run_upsampler_micro(args, dev, timeit, peaks):
    """The shipped latent upsampler (configs/latent_upsampler_flash.yaml: 48
    channels, mid 128, 8 blocks, x2, replicate memory) on a 2K clip's LR latent
    (33 frames of 36 x 64 -> 72 x 128), seeded weights: the B200 forward against
    the reference's ops on cuDNN, same box, L2 flushed between runs."""
    up = importlib.import_module("dreamx-creator_b200.upsampler")
    T, H, W = (int(v) for v in (args.shape or "33,36,64").split(","))
    kw = dict(in_channels=48, out_channels=48, mid_channels=128, num_blocks=8, upsample_scale=2)
    sd = up.FlashLatentUpsampler.seeded_state_dict(**kw, seed=0)
    m = up.FlashLatentUpsampler(sd, **kw, memory_init="replicate", device=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(1, 48, T, H, W, device=dev, generator=g).to(torch.bfloat16)
    ms = timeit(lambda: m(x))
    sdd = {k: v.to(dev) for k, v in sd.items()}
    ref = timeit(lambda: cudnn_upsampler(sdd, x, num_blocks=8, scale=2))
    a, b = m(x).float(), cudnn_upsampler(sdd, x, num_blocks=8, scale=2).float()
    fl = m.flops(T, H, W)
    srdit_ops = importlib.import_module("dreamx-creator_b200.ops")
    srdit_ops.Stats.events = []
    m(x)
    torch.cuda.synchronize()
    evs, srdit_ops.Stats.events = srdit_ops.Stats.events, None
    conv_ms = sum(e0.elapsed_time(e1) for _, e0, e1, _ in evs)
    by_work = {}
    for _, e0, e1, wk in evs:
        k = by_work.setdefault(wk, [0, 0.0])
        k[0] += 1
        k[1] += e0.elapsed_time(e1)
    return {"workload": "FlashLatentUpsampler x2 (48 ch, mid 128, 8 blocks, replicate), "
                        f"LR latent 1 x 48 x {T} x {H} x {W}", "ms": ms,
            "latent_frames_per_s": T / ms * 1e3, "tflops": fl / ms / 1e9,
            "conv_launches": len(evs), "conv_ms": conv_ms, "conv_tflops": fl / conv_ms / 1e9,
            "frac_of_bf16_burst": fl / conv_ms / 1e9 / peaks["bf16_tflops"],
            "cudnn_ms": ref, "cudnn_tflops": fl / ref / 1e9, "speedup_vs_cudnn": ref / ms,
            "rel_fro_vs_cudnn": float((a - b).norm() / b.norm()),
            "conv_by_work": [{"gflop": wk / 1e9, "launches": n, "ms": t,
                              "tflops": wk * n / t / 1e9}
                             for wk, (n, t) in sorted(by_work.items(), reverse=True)]}


def run_vae_micro(args, dev, peaks):
    """The Wan2.2 VAE decode (dec_dim 256, z 48) of a latent [48, T, h, w]
    (default 2 frames of a 2K clip, 72 x 128 -> 5 frames of 1152 x 2048),
    seeded weights: wall time per decode (CUDA events), output frames/s, the
    algorithmic FLOP rate, and the share of the conv kernels."""
    vae = importlib.import_module("dreamx-creator_b200.vae")
    srdit_ops = importlib.import_module("dreamx-creator_b200.ops")
    T, h, w = (int(v) for v in (args.shape or "2,72,128").split(","))
    sd = vae.Wan22VAEDecoder.seeded_state_dict(seed=0)
    d = vae.Wan22VAEDecoder(sd, device=dev)
    g = torch.Generator(device=dev).manual_seed(2)
    z = torch.randn(48, T, h, w, device=dev, generator=g)
    mean, std = torch.zeros(48), torch.ones(48)
    for _ in range(1):
        d.decode(z, mean, std)
    torch.cuda.synchronize()
    ts = []
    for _ in range(max(1, args.iters)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        v = d.decode(z, mean, std)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ms = statistics.median(ts)
    srdit_ops.Stats.events = []
    d.decode(z, mean, std)
    torch.cuda.synchronize()
    evs, srdit_ops.Stats.events = srdit_ops.Stats.events, None
    per_kind = {}
    for kind, e0, e1, work in evs:
        k = per_kind.setdefault(kind, [0, 0.0, 0])
        k[0] += 1
        k[1] += e0.elapsed_time(e1)
        k[2] += work
    fl = d.flops(T, h, w)
    conv = per_kind.get("conv3d", [0, 0.0, 0])
    # the conv launches grouped by their work (one group per layer shape)
    shapes = {}
    for kind, e0, e1, work in evs:
        if kind == "conv3d":
            k = shapes.setdefault(work, [0, 0.0])
            k[0] += 1
            k[1] += e0.elapsed_time(e1)
    by_shape = sorted(((t, n, wk) for wk, (n, t) in shapes.items()), reverse=True)[:12]
    return {"workload": f"Wan2.2 VAE decode (dec_dim 256, z 48), latent 48 x {T} x {h} x {w} "
                        f"-> {tuple(v.shape)}", "ms": ms,
            "frames_per_s": v.shape[1] / ms * 1e3, "tflops": fl / ms / 1e9,
            "conv3d": {"launches": conv[0], "ms": conv[1], "tflops": conv[2] / conv[1] / 1e9,
                       "frac_of_bf16_burst": conv[2] / conv[1] / 1e9 / peaks["bf16_tflops"]},
            "kernels": {k: {"launches": n, "ms": t} for k, (n, t, _) in per_kind.items()},
            "conv3d_by_work": [{"gflop": wk / 1e9, "launches": n, "ms": t,
                                "tflops": wk * n / t / 1e9} for t, n, wk in by_shape]}


def dist_setup(n):
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 under torchrun")
    if world > 1:
        import datetime
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        torch.distributed.init_process_group(
            "nccl" if torch.cuda.is_available() else "gloo",
            timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def geometry(name):
    return ((8, 8), (0, 0)) if name == "8x8r0" else ((4, 4), (3, 3))


# --------------------------------------------------------------------------- CPU arm
_REF_BLOCK = {}


def reference_block(args):
    """The reference's own WanAttentionBlock (models.py:1207-1354) at full size,
    from its install under baseline/_ref: bf16 weights (seeded, built once),
    window attention on its CPU gather + SDPA backend (attention.py:660-802).
    None when the reference is not installed."""
    if not (REF_INSTALL / "wan" / "modules" / "sr_dit" / "models.py").exists():
        return None
    key = args.geometry
    if key in _REF_BLOCK:
        return _REF_BLOCK[key]
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    import warnings
    warnings.filterwarnings("ignore")
    from wan.modules.sr_dit import models
    D, F = 3072, 14336
    blk = models.WanAttentionBlock("t2v_cross_attn", D, F, 24, (-1, -1), True, True, 1e-6,
                                   stream_chunk_size=3)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if name.endswith("bias"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.01)
            elif "norm" in name:
                p.fill_(1.0)
            elif name == "modulation":
                p.copy_(torch.randn(p.shape, generator=g) / D ** 0.5)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    blk = blk.to(torch.bfloat16)
    blk.modulation.data = blk.modulation.data.float()
    bhw, rhw = geometry(args.geometry)
    sa = blk.self_attn
    sa.use_window_attn, sa.window_attn_impl = True, "sdpa"
    sa.window_block_hw, sa.window_block_radius_hw = bhw, rhw
    t, hd, wd = models._rope_axis_dims(128)
    freqs = torch.cat([models.rope_params(1024, t), models.rope_params(1024, hd),
                       models.rope_params(1024, wd)], dim=1)
    _REF_BLOCK[key] = (blk, freqs)
    return _REF_BLOCK[key]


def cpu_block_sample(args, seed=0):
    """Time one full-size SR-DiT block of the denoise forward (3 frames of 36 x 64
    tokens over a 3-frame cache, 512 text tokens) on the host cores.

    With the reference installed under baseline/_ref this runs the reference's
    own WanAttentionBlock.forward (kind "reference"); otherwise the oracle's
    restatement of it (bf16 Linears, fp32 window softmax; kind "port").
    Returns (seconds, threads, kind)."""
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    D, L = 3072, 36 * 64
    ref = reference_block(args)
    if ref is not None:
        blk, freqs = ref
        x = torch.randn(1, 3 * L, D, generator=g).to(torch.bfloat16)
        e = torch.randn(1, 6, D, generator=g) * 0.1
        ctx = torch.randn(1, 512, D, generator=g).to(torch.bfloat16)
        ck = torch.randn(1, 3 * L, 24, 128, generator=g).to(torch.bfloat16)
        cv = torch.randn(1, 3 * L, 24, 128, generator=g).to(torch.bfloat16)
        t0 = time.perf_counter()
        with torch.no_grad():
            blk(x, e=e, seq_lens=torch.tensor([3 * L]), grid_sizes=torch.tensor([[3, 36, 64]]),
                freqs=freqs, context=ctx, context_lens=None, temporal_offset=3, is_stream=True,
                pre_cache_k=ck, pre_cache_v=cv, kv_len=9)
        return time.perf_counter() - t0, torch.get_num_threads(), "reference"
    from oracle import block as oblock
    from oracle import numerics as onum
    F = 14336
    r = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16)  # noqa: E731
    wts = {}
    for m in ("self_attn", "cross_attn"):
        for n in ("q", "k", "v", "o"):
            wts[f"{m}.{n}.weight"], wts[f"{m}.{n}.bias"] = r(D, D), r(D)
        wts[f"{m}.norm_q.weight"] = torch.ones(D, dtype=torch.bfloat16)
        wts[f"{m}.norm_k.weight"] = torch.ones(D, dtype=torch.bfloat16)
    wts["norm3.weight"], wts["norm3.bias"] = torch.ones(D, dtype=torch.bfloat16), r(D)
    wts["ffn.0.weight"], wts["ffn.0.bias"] = r(F, D), r(F)
    wts["ffn.2.weight"], wts["ffn.2.bias"] = r(D, F), r(D)
    wts["modulation"] = torch.randn(1, 6, D, generator=g) / D ** 0.5
    x = torch.randn(3 * L, D, generator=g).to(torch.bfloat16)
    ctx = torch.randn(512, D, generator=g).to(torch.bfloat16)
    ck = torch.randn(3 * L, 24, 128, generator=g).to(torch.bfloat16)
    cv = torch.randn(3 * L, 24, 128, generator=g).to(torch.bfloat16)
    e0 = torch.randn(6, D, generator=g) * 0.1
    bhw, rhw = geometry(args.geometry)
    freqs = onum.rope_freqs()
    t0 = time.perf_counter()
    with torch.no_grad():
        oblock.block_forward(wts, x, e0, ctx, grid=(3, 36, 64), freqs=freqs, t_offset=3,
                             cache_k=ck, cache_v=cv, kv_len=9, block_hw=bhw, radius_hw=rhw,
                             block_t=3, heads=24, linear="bf16")
    return time.perf_counter() - t0, torch.get_num_threads(), "port"


CPU_SAMPLE = {
    "reference": "the reference's own WanAttentionBlock.forward (bf16 Linears, window "
                 "attention on its CPU gather + SDPA backend)",
    "port": "the CPU restatement of WanAttentionBlock (bf16 Linears, fp32 window softmax)",
}


def cpu_value(block_s, layers=30):
    # a step is 2 forwards x `layers` blocks (embeddings / head are < 1% and omitted)
    return FRAMES_PER_STEP / (2 * layers * block_s)


def run_reference_arm(args, rank):
    if rank != 0:
        return
    times = []
    cores = 1
    kind = "port"
    for i in range(args.warmup + args.steps):
        t, cores, kind = cpu_block_sample(args, seed=i)
        if i >= args.warmup:
            times.append(t)
    blk = statistics.mean(times)
    val = cpu_value(blk)
    # each step timed here is the bounded sample (one block); the metric's value
    # scales it to the 60 block-forwards of a refinement chunk
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * blk, "sample_unit": "one full-size block per step",
            "chunk_ms_extrapolated": 1e3 * FRAMES_PER_STEP / val, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"one full-size SR-DiT block per step: {CPU_SAMPLE[kind]}; "
                                       f"x60 for the 2-forward chunk"},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm
def workload_config(args):
    bhw, rhw = geometry(args.geometry)
    return {"workload": "config3: SR-DiT 5B 2K AR chunk (denoise t=625 + KV refresh t=0), "
                        "3 latent frames 36x64 tokens, 3-frame KV prefix, 512 text tokens",
            "model": "SR-DiT 5B (30 blocks, dim 3072, 24x128 heads, ffn 14336)",
            "layers": args.layers, "tokens": 6912, "window": f"3x{bhw[0]}x{bhw[1]} r{rhw}",
            "global_batch": args.gpus if args.parallel == "replicas" else 1, "seq_len": 6912,
            "parallelism": ({"tp": f"tp{args.gpus} (sequence-parallel residual stream, "
                                   f"{args.tp_comm} collectives)",
                             "spatial": f"spatial{args.gpus} (w-strips of whole windows, "
                                        f"full model per GPU, one all-gather per forward"
                                        f"{'; K/V halo by ' + args.halo if args.geometry != '8x8r0' else ''})",
                             "replicas": "replicas"}[args.parallel]) if args.gpus > 1
            else "single",
            "l2": "inputs larger than L2 (5 GB of fp8 weights stream every forward)",
            "lq_anchor": {"none": "off",
                          "serial": "frame-aligned, harvested inside every step (3 forwards)",
                          "overlap": "frame-aligned, next step's harvest on a side stream "
                                     "(3 forwards)"}[args.anchor]}


class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = pathlib.Path(f"/tmp/srdit_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.f.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return None
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
                for n, v in zip(names, r[4:8]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def run_gpu_arm(args, rank, world, local):
    srdit = importlib.import_module("dreamx-creator_b200")
    from importlib import import_module
    model_mod = import_module("dreamx-creator_b200.model")
    pipe_mod = import_module("dreamx-creator_b200.pipeline")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    bhw, rhw = geometry(args.geometry)
    cfg = model_mod.SRDiTConfig(num_layers=args.layers, block_hw=bhw, block_radius_hw=rhw)
    tp = world > 1 and args.parallel in ("tp", "spatial")   # one clip over all ranks
    if world > 1 and args.parallel == "tp":
        tp_mod = import_module("dreamx-creator_b200.tp")
        model = tp_mod.TPSRDiT.random_init(cfg, dev, seed=0, fused=args.tp_comm == "fused")
    elif world > 1 and args.parallel == "spatial":
        sp_mod = import_module("dreamx-creator_b200.spatial")
        model = sp_mod.SpatialSRDiT.random_init(cfg, dev, seed=0, halo=args.halo)
    else:
        model = model_mod.SRDiT.random_init(cfg, dev, seed=0)
    # tensor parallelism refines one clip on all ranks; replicas one clip each
    g = torch.Generator().manual_seed(1000 if tp else 1000 + rank)
    ctx_host = torch.randn(*CTX_SHAPE, generator=g).to(torch.bfloat16).pin_memory()
    noisy_host = torch.randn(*LAT_SHAPE, generator=g).to(torch.bfloat16).pin_memory()
    prefix_host = torch.randn(*LAT_SHAPE, generator=g).to(torch.bfloat16).pin_memory()
    out_host = torch.empty(*LAT_SHAPE, dtype=torch.bfloat16).pin_memory()
    ctx = ctx_host.to(dev)
    noisy = noisy_host.to(dev)
    stream = pipe_mod.RefinerStream(model, ctx, graphs=not args.no_graphs)
    # prefill: the previous chunk's refresh forward leaves a 3-frame cache
    stream.step(prefix_host.to(dev))
    ring = stream.cache
    prefix_state = (ring.start, ring.frames, stream.t_offset)

    lq_host = torch.randn(*LAT_SHAPE, generator=g).to(torch.bfloat16).pin_memory()
    lq = lq_host.to(dev)

    def one_step(inp):
        ring.start, ring.frames, stream.t_offset = prefix_state
        if args.anchor == "none":
            return stream.step(inp)
        if args.anchor == "serial":
            return stream.step(inp, lq_chunk=lq)
        # the next step's anchor (same temporal position: the ring is reset to
        # the prefix every step) is harvested on the side stream meanwhile
        return stream.step(inp, lq_chunk=lq, next_lq_chunk=lq, next_t_offset=prefix_state[2])

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad():
        ops = srdit.ops
        with ClockSampler(local) as clk:   # samples warm-up and the timed region
            for _ in range(args.warmup):
                one_step(noisy)
            stream.check_status()
            barrier()
            # ---- device-timed region: inputs resident in HBM, nothing but the steps
            l0 = ops.Stats.launches
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.nvtx.range_push("srdit_step")
            e0.record()
            h0 = time.perf_counter()
            for _ in range(args.steps):
                one_step(noisy)
            host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # issuing only
            e1.record()
            torch.cuda.nvtx.range_pop()
            barrier()
        replayed = ops.Stats.launches - l0   # 0 when the steps replay a graph
        dev_ms = max_over_ranks(e0.elapsed_time(e1))
        stream.check_status()
        # ---- attribution pass (outside the timed region): one more step with CUDA
        # events around every launch on the launching stream
        ops.Stats.events = []
        graphs, stream.graphs = stream.graphs, False
        l1 = ops.Stats.launches
        one_step(noisy)
        launches_per_step = ops.Stats.launches - l1
        stream.graphs = graphs
        torch.cuda.synchronize()
        kinds = {}
        for kind, a, b, work in ops.Stats.events:
            k = kinds.setdefault(kind, [0, 0.0, 0])
            k[0] += 1
            k[1] += a.elapsed_time(b)
            k[2] += work
        ops.Stats.events = None
        # ---- end-to-end region: the public API with host buffers
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            c = ctx_host.to(dev, non_blocking=True)
            stream.set_context(c)
            x = noisy_host.to(dev, non_blocking=True)
            if args.anchor != "none":
                lq.copy_(lq_host, non_blocking=True)
            y = one_step(x)
            out_host.copy_(y, non_blocking=True)
        s1.record()
        barrier()
        e2e_ms = max_over_ranks(s0.elapsed_time(s1))
        stream.set_context(ctx)

    if rank != 0:
        return
    peaks, peak_kind = load_peaks()
    fp8_peak = 2.0 * float(peaks.get("bf16_tflops_sustained", 1400.0))
    bf16_peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    clips = 1 if tp else world   # clips refined per step, over all ranks
    value = clips * FRAMES_PER_STEP * args.steps / (dev_ms * 1e-3)
    e2e_val = clips * FRAMES_PER_STEP * args.steps / (e2e_ms * 1e-3)
    step_ms = dev_ms / args.steps
    n_gemm, gemm_ms, gemm_flop = kinds.get("fp8_gemm", [0, 0.0, 0])
    achieved = gemm_flop / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    breakdown = {}
    for kind, (n, ms, work) in sorted(kinds.items(), key=lambda kv: -kv[1][1]):
        tensor = kind in ("fp8_gemm", "winattn")
        rate = work / (ms * 1e-3) / (1e12 if tensor else 1e9) if ms > 0 else None
        peak = fp8_peak if kind == "fp8_gemm" else bf16_peak if kind == "winattn" else hbm_peak
        breakdown[kind] = {"launches": n, "ms": round(ms, 3), "share": round(ms / step_ms, 4),
                           "rate": rate, "rate_unit": "TFLOP/s" if tensor else "GB/s",
                           "frac": (rate / peak) if rate else None}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "e4m3 GEMM (fp32 acc) / bf16 attention", "data": "synthetic (seeded N(0,1) "
        "latent + text context, seeded random weights)",
        "config": workload_config(args),
        "roofline": {"bound": "tensor", "kernel": "srdit_fp8_gemm (tcgen05 e4m3)",
                     "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": (achieved / fp8_peak) if achieved else None,
                     "traffic": GEMM_TRAFFIC_PER_LAUNCH,
                     "algorithmic_flop_per_launch": gemm_flop / max(n_gemm, 1),
                     "peak_source": f"2 x bf16_tflops_sustained of MEASURED_PEAKS.json "
                                    f"({peak_kind}); e4m3 tcgen05 rate = 2 x bf16",
                     "launches_per_step": n_gemm, "ms_per_step": gemm_ms},
        "kernels": breakdown,
        "e2e": {"value": e2e_val, "unit": UNIT,
                "h2d_bytes_per_step": noisy_host.numel() * 2 + ctx_host.numel() * 2
                + (lq_host.numel() * 2 if args.anchor != "none" else 0),
                "d2h_bytes_per_step": out_host.numel() * 2},
        "gpu_launches": launches_per_step * args.steps,
        "cuda_graph": stream.graphs and replayed == 0,
        "host_ms_per_step": host_ms,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        t, cores, kind = cpu_block_sample(args)
        line["cpu_baseline"] = {"value": cpu_value(t), "unit": UNIT, "cores": cores,
                                "kind": kind,
                                "sample": f"one full-size block on the host ({t:.2f} s): "
                                          f"{CPU_SAMPLE[kind]}; x60 for the 2-forward chunk"}
    print(json.dumps(line), flush=True)


def run_clip(args, rank, world, local):
    """Config 5: 121 video frames -> 31 latent frames, padded to 33 (the
    reference pads the latent length to whole chunks, inference_sr.py:896-903)
    -> 11 three-frame chunks through RefinerStream with kv_len 9 (f_kv 3, 6, 9,
    12, 12, ...). Two untimed passes over the clip warm up and capture the
    step's CUDA graphs (one per ring phase); the third pass is timed chunk by
    chunk with CUDA events (max over ranks). VAE decode is excluded."""
    from importlib import import_module
    import_module("dreamx-creator_b200")
    model_mod = import_module("dreamx-creator_b200.model")
    pipe_mod = import_module("dreamx-creator_b200.pipeline")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    bhw, rhw = geometry(args.geometry)
    cfg = model_mod.SRDiTConfig(num_layers=args.layers, block_hw=bhw, block_radius_hw=rhw)
    tp = world > 1 and args.parallel in ("tp", "spatial")   # one clip over all ranks
    if world > 1 and args.parallel == "tp":
        tp_mod = import_module("dreamx-creator_b200.tp")
        model = tp_mod.TPSRDiT.random_init(cfg, dev, seed=0, fused=args.tp_comm == "fused")
    elif world > 1 and args.parallel == "spatial":
        sp_mod = import_module("dreamx-creator_b200.spatial")
        model = sp_mod.SpatialSRDiT.random_init(cfg, dev, seed=0, halo=args.halo)
    else:
        model = model_mod.SRDiT.random_init(cfg, dev, seed=0)
    n_chunks, f = 11, 3
    if args.pipeline:
        if world > 1:
            raise SystemExit("--pipeline runs on one GPU")
        return run_pipeline(args, model, dev, n_chunks, f)
    g = torch.Generator().manual_seed(1000 if tp else 1000 + rank)
    ctx = torch.randn(*CTX_SHAPE, generator=g).to(torch.bfloat16).to(dev)
    clip = torch.randn(48, n_chunks * f, 72, 128, generator=g).to(torch.bfloat16).to(dev)
    stream = pipe_mod.RefinerStream(model, ctx, graphs=not args.no_graphs)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor(v, device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return t.tolist()

    with torch.no_grad():
        for _ in range(2):
            stream.reset()
            for i in range(n_chunks):
                stream.step(clip[:, i * f:(i + 1) * f])
        torch.cuda.synchronize()
        model.check_status()
        if world > 1:
            torch.distributed.barrier()
        stream.reset()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_chunks + 1)]
        evs[0].record()
        for i in range(n_chunks):
            stream.step(clip[:, i * f:(i + 1) * f])
            evs[i + 1].record()
        torch.cuda.synchronize()
        model.check_status()
    lat = max_over_ranks([evs[i].elapsed_time(evs[i + 1]) for i in range(n_chunks)])
    if rank != 0:
        return
    total = sum(lat)
    srt = sorted(lat)
    pct = lambda q: srt[min(len(srt) - 1, int(round(q * (len(srt) - 1))))]  # noqa: E731
    print(json.dumps({
        "metric": "2K long-clip refine latent-frames/s (config 5: 121 frames, 11 AR chunks)",
        "value": n_chunks * f / (total * 1e-3), "unit": UNIT, "n_gpus": world,
        "higher_is_better": True, "scaling": "strong" if tp else "weak",
        "chunk_ms": lat, "p50_ms": pct(0.5), "p99_ms": pct(0.99),
        "cuda_graph": bool(stream.graphs), "config": workload_config(args),
        "data": "synthetic (seeded N(0,1) latent clip + text context, seeded random weights)"}),
        flush=True)


def run_pipeline(args, model, dev, n_chunks, f):
    """One 121-frame 2K clip through the latent path (seeded weights, synthetic LR
    latent): FlashLatentUpsampler (the shipped config) 36 x 64 -> 72 x 128, the
    noise mix at t = 625, 11 refiner chunks (graph replay, as in config 5), the
    Wan2.2 VAE decode of the 33 refined latent frames to 129 frames of 1152 x
    2048. One untimed pass, then one timed with CUDA events between stages."""
    from importlib import import_module
    pipe_mod = import_module("dreamx-creator_b200.pipeline")
    up_mod = import_module("dreamx-creator_b200.upsampler")
    vae_mod = import_module("dreamx-creator_b200.vae")
    kw = dict(in_channels=48, out_channels=48, mid_channels=128, num_blocks=8, upsample_scale=2)
    up = up_mod.FlashLatentUpsampler(up_mod.FlashLatentUpsampler.seeded_state_dict(**kw),
                                     **kw, memory_init="replicate", device=dev)
    dec = vae_mod.Wan22VAEDecoder(vae_mod.Wan22VAEDecoder.seeded_state_dict(seed=0), device=dev)
    T = n_chunks * f
    g = torch.Generator(device=dev).manual_seed(1000)
    ctx = torch.randn(*CTX_SHAPE, device=dev, generator=g).to(torch.bfloat16)
    lr = torch.randn(1, 48, T, 36, 64, device=dev, generator=g).to(torch.bfloat16)
    noise = torch.randn(48, T, 72, 128, device=dev, generator=g).to(torch.bfloat16)
    mean, std = torch.zeros(48), torch.ones(48)
    stream = pipe_mod.RefinerStream(model, ctx, graphs=not args.no_graphs)
    sigma = stream.denoise_t / stream.ntt

    def once(evs):
        evs[0].record()
        lr_up = up(lr)[0]
        evs[1].record()
        noisy = pipe_mod.sr_noise(lr_up, noise, sigma)
        stream.reset()
        x0 = pipe_mod.refine_clip(stream, noisy, chunk=f)
        evs[2].record()
        video = dec.decode(x0, mean, std)
        evs[3].record()
        return video

    with torch.no_grad():
        once([torch.cuda.Event(enable_timing=True) for _ in range(4)])
        torch.cuda.synchronize()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        video = once(evs)
        torch.cuda.synchronize()
        model.check_status()
    st = [evs[i].elapsed_time(evs[i + 1]) for i in range(3)]
    total = sum(st)
    print(json.dumps({
        "metric": "2K clip latent path seconds (upsample + 11-chunk refine + VAE decode)",
        "value": total * 1e-3, "unit": "s", "n_gpus": 1, "higher_is_better": False,
        "stages_ms": {"latent_upsampler": st[0], "refine_11_chunks": st[1], "vae_decode": st[2]},
        "video": list(video.shape), "output_frames_per_s": video.shape[1] / (total * 1e-3),
        "cuda_graph": bool(stream.graphs),
        "data": "synthetic (seeded N(0,1) LR latent, noise and text context; seeded random "
                "weights for the upsampler, the refiner and the VAE decoder)"}), flush=True)


def main():
    args = parse()
    if args.micro:
        return run_micro(args)
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference_arm(args, rank)
        elif args.clip:
            run_clip(args, rank, world, local)
        else:
            run_gpu_arm(args, rank, world, local)
    finally:
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
