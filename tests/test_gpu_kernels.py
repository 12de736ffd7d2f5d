"""Parity of the sm_100a kernels with the CPU oracle (GPU required)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import blockgrid as obg
from oracle import numerics as onum
from oracle import winattn as owa
from tests.golden_cases import config1_inputs, stream_inputs

pytestmark = pytest.mark.gpu


def _bf16_bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy()


# --------------------------------------------------------------------------- quantiser
@pytest.mark.parametrize("M,K", [(64, 512), (300, 3072), (7, 14336), (4096, 3072)])
def test_quant_rowwise_bit_exact(srdit, cuda_device, M, K):
    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(M, K, generator=g)
    x = torch.where(torch.rand(M, K, generator=g) < 1e-3, x * 20, x).to(torch.bfloat16)
    x[M // 2] = 0
    q, s = srdit.ops.quant_rowwise(x.to(cuda_device))
    qo, so = onum.quantize_rowwise(x)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), qo.view(torch.uint8).numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), so.reshape(-1).numpy())
    # with a precomputed amax the single-pass path gives the same bytes
    amax = x.float().abs().amax(-1).to(cuda_device)
    q2, s2 = srdit.ops.quant_rowwise(x.to(cuda_device), amax=amax)
    assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8)) and torch.equal(s2, s)


@pytest.mark.parametrize("affine,modulate", [(False, True), (True, False), (False, False)])
def test_ln_mod_quant(srdit, cuda_device, affine, modulate):
    M, K = 200, 3072
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(M, K, generator=g) * 2 + 0.3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16) if affine else None
    b = (0.1 * torch.randn(K, generator=g)).to(torch.bfloat16) if affine else None
    shift = (0.1 * torch.randn(K, generator=g)) if modulate else None
    scale = (0.1 * torch.randn(K, generator=g)) if modulate else None
    dev = lambda t: None if t is None else t.to(cuda_device)  # noqa: E731
    q, qs = srdit.ops.ln_mod_quant(dev(x), 1e-6, ln_weight=dev(w), ln_bias=dev(b),
                                   shift=dev(shift), scale=dev(scale))
    n = onum.layer_norm(x, 1e-6, w, b)
    if modulate:
        n = (n.float() * (1 + scale) + shift).to(torch.bfloat16)
    qo, so = onum.quantize_rowwise(n)
    # LayerNorm statistics are reduced in a different order than torch's CPU
    # kernel, so a bf16 tie can round the other way before quantisation. Measured
    # on B200 (this test's inputs and 6912 x 3072, 4096 x 4096, 2000 x 1024 with
    # each mode): 0 to 1.6e-6 of the e4m3 bytes differ, every row scale is
    # bit-identical; the bounds below keep an order of magnitude of margin.
    deq = q.float().cpu() * qs.cpu()[:, None]
    deq_o = qo.float() * so
    assert onum.rel_fro(deq, deq_o) < 1e-4
    assert (q.view(torch.uint8).cpu() != qo.view(torch.uint8)).float().mean() <= 1e-5
    np.testing.assert_array_equal(qs.cpu().numpy(), so.reshape(-1).numpy())


def test_rms_rope_matches_reference_math(srdit, cuda_device):
    f, h, w, n = 2, 5, 7, 24
    K = n * 128
    M = f * h * w
    g = torch.Generator().manual_seed(9)
    src = torch.randn(M, 3 * K, generator=g).to(torch.bfloat16)   # fused [q | k | v] rows
    wq = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    freqs = onum.rope_freqs()
    cos, sin = onum.rope_tables(freqs)
    d_src = src.to(cuda_device)
    q_out = torch.empty(M, K, dtype=torch.bfloat16, device=cuda_device)
    # K/V into a 4-frame ring starting at slot 3 (frames land in slots 3, 0)
    k_ring = torch.zeros(4 * h * w, K, dtype=torch.bfloat16, device=cuda_device)
    v_ring = torch.zeros_like(k_ring)
    srdit.ops.rms_rope(d_src[:, :K], wq.to(cuda_device), 1e-6, q_out, frame_tokens=h * w,
                       cos=cos.to(cuda_device), sin=sin.to(cuda_device), grid_h=h, grid_w=w,
                       t_offset=4)
    srdit.ops.rms_rope(d_src[:, K:2 * K], wq.to(cuda_device), 1e-6, k_ring, frame_tokens=h * w,
                       slot0=3, n_slots=4, cos=cos.to(cuda_device), sin=sin.to(cuda_device),
                       grid_h=h, grid_w=w, t_offset=4, v_src=d_src[:, 2 * K:], v_dst=v_ring)
    ref_q = onum.rope_apply(onum.rms_norm(src[:, :K], wq).view(M, n, 128), (f, h, w), freqs, 4)
    ref_k = onum.rope_apply(onum.rms_norm(src[:, K:2 * K], wq).view(M, n, 128), (f, h, w),
                            freqs, 4)
    got_q = q_out.cpu().view(M, n, 128)
    # mean() is reduced in another order than torch's CPU kernel: rare 1-ulp ties
    assert (got_q.view(torch.int16) == ref_q.view(torch.int16)).float().mean() > 0.99
    assert onum.rel_fro(got_q.float(), ref_q.float()) < 1e-3
    L = h * w
    ring = k_ring.cpu()
    got_k = torch.cat([ring[3 * L:4 * L], ring[0:L]]).view(M, n, 128)
    assert onum.rel_fro(got_k.float(), ref_k.float()) < 1e-3
    vr = v_ring.cpu()
    assert torch.equal(torch.cat([vr[3 * L:4 * L], vr[0:L]]), src[:, 2 * K:])
    assert ring[L:3 * L].abs().sum() == 0  # untouched slots stay untouched


# --------------------------------------------------------------------------- fp8 GEMM
def _gemm_inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    a = torch.where(torch.rand(M, K, generator=g) < 1e-3, a * 20, a).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    aq, as_ = onum.quantize_rowwise(a)
    wq, ws = onum.fp8_linear_weights(w)
    return a, aq, as_.reshape(-1).contiguous(), wq, ws, bias


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 320, 640), (512, 3072, 3072),
                                   (130, 9216, 256)])
def test_fp8_gemm_store(srdit, cuda_device, M, N, K):
    a, aq, as_, wq, ws, bias = _gemm_inputs(M, N, K, M * 7 + N)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    out = srdit.ops.fp8_gemm(d(aq), d(as_), d(wq), d(ws), d(bias))
    ref = onum.fp8_linear(a, wq, ws, bias)
    assert onum.rel_fro(out.cpu().float(), ref.float()) < 1e-3
    # against the reference's own GPU call (cuBLASLt row-wise torch._scaled_mm)
    if K % 16 == 0 and N % 16 == 0:
        sm = torch._scaled_mm(d(aq), d(wq).t(), scale_a=d(as_).view(-1, 1),
                              scale_b=d(ws).view(1, -1), bias=d(bias), out_dtype=torch.bfloat16)
        assert onum.rel_fro(out.float(), sm.float()) < 1e-3


def test_fp8_gemm_gelu_amax(srdit, cuda_device):
    M, N, K = 256, 1024, 512
    a, aq, as_, wq, ws, bias = _gemm_inputs(M, N, K, 11)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    amax = torch.zeros(M, device=cuda_device)
    out = srdit.ops.fp8_gemm(d(aq), d(as_), d(wq), d(ws), d(bias), epilogue="gelu",
                             row_amax=amax)
    ref = onum.gelu_tanh(onum.fp8_linear(a, wq, ws, bias))
    assert onum.rel_fro(out.cpu().float(), ref.float()) < 2e-3
    np.testing.assert_array_equal(amax.cpu().numpy(), out.float().abs().amax(-1).cpu().numpy())


@pytest.mark.parametrize("kind", ["gated_res", "res"])
def test_fp8_gemm_residual(srdit, cuda_device, kind):
    M, N, K = 384, 512, 768
    a, aq, as_, wq, ws, bias = _gemm_inputs(M, N, K, 13)
    g = torch.Generator().manual_seed(14)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    gate = torch.randn(N, generator=g) * 0.5
    d = lambda t: t.to(cuda_device)  # noqa: E731
    out = srdit.ops.fp8_gemm(d(aq), d(as_), d(wq), d(ws), d(bias), epilogue=kind,
                             residual=d(res), gate=d(gate) if kind == "gated_res" else None)
    y = onum.fp8_linear(a, wq, ws, bias)
    ref = (res.float() + y.float() * gate) if kind == "gated_res" else (res.float() + y.float())
    ref = ref.to(torch.bfloat16)
    assert onum.rel_fro(out.cpu().float(), ref.float()) < 1e-3


@pytest.mark.parametrize("kind", ["gated_res", "res"])
def test_fp8_gemm_residual_in_place_ragged(srdit, cuda_device, kind):
    """The block's use: the output overwrites the residual stream it reads
    (out is residual), here with M and N that end inside a 32 x 64 residual box
    and an output-tile pair; 10 x 8 tiles, so some CTA pairs take two (the
    residual box of a pair's next tile is loaded during its current one)."""
    M, N, K = 2536, 1480, 256
    a, aq, as_, wq, ws, bias = _gemm_inputs(M, N, K, 23)
    g = torch.Generator().manual_seed(24)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    gate = torch.randn(N, generator=g) * 0.5
    d = lambda t: t.to(cuda_device)  # noqa: E731
    x = d(res)
    out = srdit.ops.fp8_gemm(d(aq), d(as_), d(wq), d(ws), d(bias), x, epilogue=kind, residual=x,
                             gate=d(gate) if kind == "gated_res" else None)
    assert out.data_ptr() == x.data_ptr()
    y = onum.fp8_linear(a, wq, ws, bias)
    ref = (res.float() + y.float() * gate) if kind == "gated_res" else (res.float() + y.float())
    ref = ref.to(torch.bfloat16)
    assert onum.rel_fro(x.cpu().float(), ref.float()) < 1e-3
    assert (x.cpu().view(torch.int16) == ref.view(torch.int16)).float().mean() > 0.99


# --------------------------------------------------------------------------- window attention
def _check_attn(got, ref, max_abs=2e-2, rel=5e-3):
    got = got.float().cpu().double()
    ref = ref.double()
    err = (got - ref).abs().max().item()
    r = onum.rel_fro(got, ref)
    assert err <= max_abs and r <= rel, (err, r)
    return err, r


@pytest.mark.parametrize("bhw,rhw", [((8, 8), (0, 0)), ((4, 4), (3, 3))])
def test_winattn_config1(srdit, cuda_device, golden, bhw, rhw):
    """BASELINE config 1 (3x18x32 grid, 24 heads, RoPE'd N(0,1) q/k/v, seed 0)."""
    qr, kr, v = config1_inputs()
    qb, kb, vb = (t.to(torch.bfloat16) for t in (qr, kr, v))
    out, _, _ = srdit.attention.mask_free_window_attention(
        qb[None].to(cuda_device), kb[None].to(cuda_device), vb[None].to(cuda_device),
        torch.tensor([[3, 18, 32]]), attn_impl="b200", block_t=3, block_hw=bhw,
        block_radius_hw=rhw)
    spec = obg.make_spec(3, 3, 18, 32, block_t=3, block_hw=bhw, block_radius_hw=rhw)
    ref = owa.run_plan(qb, kb, vb, obg.build_plan(spec), f_cur=3, h=18, w=32)
    _check_attn(out[0], ref)
    # and against the reference's own fp32 output (bf16 input rounding included)
    tag = "cfg1_%dx%d_r%d" % (bhw[0], bhw[1], rhw[0])
    gold = torch.from_numpy(golden("winattn")[f"{tag}.out_h0"])
    _check_attn(out[0, :, 0], gold, max_abs=3e-2, rel=1e-2)


@pytest.mark.parametrize("tag", ["none", "frame", "chunk"])
def test_winattn_streaming_cache_anchor(srdit, cuda_device, tag):
    ins = {k: v.to(torch.bfloat16) for k, v in stream_inputs().items()}
    d = lambda t: t[None].to(cuda_device)  # noqa: E731
    kw = {} if tag == "none" else dict(anchor_k=d(ins["ak"]), anchor_v=d(ins["av"]),
                                       anchor_align=tag)
    out, nck, ncv = srdit.attention.mask_free_window_attention(
        d(ins["q"]), d(ins["k"]), d(ins["v"]), torch.tensor([[3, 8, 12]]),
        pre_cache_k=d(ins["ck"]), pre_cache_v=d(ins["cv"]), kv_len=4, attn_impl="b200",
        block_t=3, block_hw=(4, 4), block_radius_hw=(1, 1), **kw)
    spec = obg.make_spec(3, 6, 8, 12, block_t=3, block_hw=(4, 4), block_radius_hw=(1, 1),
                         streaming=True)
    anchor = None if tag == "none" else tag
    plan = obg.build_plan(spec, anchor)
    k_full = torch.cat([ins["ck"], ins["k"]])
    v_full = torch.cat([ins["cv"], ins["v"]])
    if anchor:
        k_full = torch.cat([ins["ak"], k_full])
        v_full = torch.cat([ins["av"], v_full])
    ref = owa.run_plan(ins["q"], k_full, v_full, plan, f_cur=3, h=8, w=12)
    _check_attn(out[0], ref)
    assert torch.equal(nck[0].cpu(), torch.cat([ins["ck"], ins["k"]])[-4 * 96:])


@pytest.mark.parametrize("geom", ["2k_4x4_r3_f12_frame", "2k_8x8_r0_f6", "odd_frame",
                                  "native_anchor", "hist_rt1", "parallel_causal"])
def test_winattn_reference_plans(srdit, cuda_device, golden, geom):
    """Launch with the reference's own params rows (the launcher seam)."""
    from tests.golden_cases import spec_fields
    g = golden("plans")
    vals, mode = spec_fields(g, geom)
    f_cur, f_kv, h, w = vals["f_cur"], vals["f_kv"], vals["h"], vals["w"]
    n = 2
    L = h * w
    ahw = vals["anchor_hw"] or (h, w)
    La = ahw[0] * ahw[1]
    gen = torch.Generator().manual_seed(21)
    q = torch.randn(f_cur * L, n, 128, generator=gen).to(torch.bfloat16)
    a_tok = f_cur * La if mode else 0
    k = torch.randn(a_tok + f_kv * L, n, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(a_tok + f_kv * L, n, 128, generator=gen).to(torch.bfloat16)
    meta = g[f"{geom}.meta"]
    plan = {"params": torch.from_numpy(g[f"{geom}.params"]), "n_w": int(meta[0]),
            "block_m": int(meta[1]), "m_tiles": int(meta[2]), "block_n": int(meta[3]),
            "hr_base": int(meta[4]), "p_stride": int(meta[5])}
    out = torch.empty_like(q, device=cuda_device)
    srdit.attention.run_blockgrid_b200(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                       out, plan=plan, f_cur=f_cur, h=h, w=w, n=n, d=128,
                                       anchor_mode=mode)
    oplan = {**plan, "params": g[f"{geom}.params"]}
    ref = owa.run_plan(q, k, v, oplan, f_cur=f_cur, h=h, w=w)
    _check_attn(out, ref)


def test_winattn_two_kv_segments_ring(srdit, cuda_device):
    """srdit_winattn_fwd with its K/V ring split over two buffers (slots below
    kv_split in the first, the rest in the second), the window's frames starting
    past the split and wrapping round the ring: the same bytes as one buffer
    holding the whole ring."""
    att = srdit.attention
    h, w, n, d = 8, 12, 2, 128
    L, f_cur, f_kv, slots, slot0, split = h * w, 3, 6, 7, 5, 4
    spec = srdit.blockgrid.make_spec(f_cur=f_cur, f_kv=f_kv, h=h, w=w, block_t=3,
                                     block_hw=(4, 4), block_radius_hw=(1, 1), streaming=True)
    plan = att.cached_plan(spec)
    g = torch.Generator().manual_seed(17)
    q = torch.randn(f_cur * L, n * d, generator=g).to(torch.bfloat16).to(cuda_device)
    ring_k = torch.randn(slots * L, n * d, generator=g).to(torch.bfloat16).to(cuda_device)
    ring_v = torch.randn(slots * L, n * d, generator=g).to(torch.bfloat16).to(cuda_device)
    params_dev, tiling, n_w, mode, split_dev = att._plan_device_state(
        plan, cuda_device, None, ("two_seg", f_kv),
        dict(f_cur=f_cur, h=h, w=w, kv_frames=f_kv, a_hw=None, a_frames=0))
    outs = []
    for two in (False, True):
        k1 = ring_k[:split * L] if two else ring_k
        v1 = ring_v[:split * L] if two else ring_v
        geo = att._geom(q, k1, f_cur=f_cur, h=h, w=w, n=n, d=d, kv_frames=slots, kv_slot0=slot0)
        geo.col_split = None if split_dev is None else split_dev.data_ptr()
        if two:
            geo.k_hr2 = ring_k[split * L:].data_ptr()
            geo.v_hr2 = ring_v[split * L:].data_ptr()
            geo.kv_split = split
        out = torch.zeros_like(q)
        srdit.ops.winattn(q, k1, v1, out, params_dev=params_dev, n_w=n_w,
                          p_stride=int(plan["p_stride"]), anchor_mode=mode, geom=geo,
                          tiling=tiling)
        outs.append(out)
    torch.cuda.synchronize()
    assert outs[0].abs().sum() > 0
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))


def test_winattn_deterministic(srdit, cuda_device):
    ins = {k: v.to(torch.bfloat16) for k, v in stream_inputs().items()}
    d = lambda t: t[None].to(cuda_device)  # noqa: E731
    outs = [srdit.attention.mask_free_window_attention(
        d(ins["q"]), d(ins["k"]), d(ins["v"]), torch.tensor([[3, 8, 12]]),
        pre_cache_k=d(ins["ck"]), pre_cache_v=d(ins["cv"]), attn_impl="b200", block_t=3,
        block_hw=(4, 4), block_radius_hw=(2, 2))[0] for _ in range(2)]
    assert torch.equal(outs[0], outs[1])


def test_fp8_gemm_v_ring(srdit, cuda_device):
    """The q|k|v GEMM with its V columns stored into ring slots: bit-identical to
    the plain GEMM's columns, frame f in slot (slot0 + f) % n_slots."""
    M, N, K, ft, cap, slot0 = 3 * 256, 3 * 384, 512, 256, 5, 3
    g = torch.Generator().manual_seed(12)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    aq, as_ = onum.quantize_rowwise(a)
    wq, ws = onum.fp8_linear_weights(w)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    plain = srdit.ops.fp8_gemm(d(aq), d(as_.reshape(-1).contiguous()), d(wq), d(ws), d(bias))
    out = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda_device)
    ring = torch.zeros(cap * ft, N - 2 * 384, dtype=torch.bfloat16, device=cuda_device)
    srdit.ops.fp8_gemm(d(aq), d(as_.reshape(-1).contiguous()), d(wq), d(ws), d(bias), out,
                       v_ring=(ring, 2 * 384, ft, slot0, cap))
    torch.cuda.synchronize()
    assert torch.equal(out[:, :768], plain[:, :768])
    assert not bool(out[:, 768:].any())   # V columns never reach out
    for f in range(M // ft):
        s = (slot0 + f) % cap
        assert torch.equal(ring[s * ft:(s + 1) * ft], plain[f * ft:(f + 1) * ft, 768:])
    used = {(slot0 + f) % cap for f in range(M // ft)}
    for s in set(range(cap)) - used:
        assert not bool(ring[s * ft:(s + 1) * ft].any())


# --------------------------------------------------------------------------- bounded waits
def test_residual_wait_times_out_into_the_status_word(srdit, cuda_device):
    """A peer flag that nothing raises: srdit_residual_tp's bounded wait runs out
    (2 s of %globaltimer), the kernel ORs SRDIT_STATUS_TIMEOUT into the status word,
    skips its rows and returns -- no hang, no trap. The context stays usable: the
    same launch with the flag raised then completes and updates x."""
    M, N = 32, 64   # one thread block
    g = torch.Generator().manual_seed(31)
    x0 = torch.randn(M, N, generator=g).to(torch.bfloat16)
    parts = torch.randn(1, M, N, generator=g).to(torch.bfloat16).to(cuda_device)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    x = x0.to(cuda_device)
    srdit.ops.residual_tp(x, parts, flags=flags.data_ptr(), expected=1, status=status)
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == srdit._lib.SRDIT_STATUS_TIMEOUT
    assert torch.equal(x.cpu(), x0)            # its rows were skipped
    flags.fill_(1)
    status.zero_()
    srdit.ops.residual_tp(x, parts, flags=flags.data_ptr(), expected=1, status=status)
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0
    ref = (x0.float() + parts[0].cpu().float()).to(torch.bfloat16)
    assert torch.equal(x.cpu(), ref)


def test_allreduce_wait_times_out_into_the_status_word(srdit, cuda_device):
    """srdit_tp_allreduce with one rank asked for epoch 2 after its first call:
    its own counter reaches only SRDIT_AR_BLOCKS (one per block), the bounded
    waits run out, the status word says so and ``out`` is left untouched. A
    second call (the counter then reaches 2 * SRDIT_AR_BLOCKS) completes and
    reduces."""
    n = 1000
    vals = torch.randn(n, generator=torch.Generator().manual_seed(32)).to(cuda_device)
    t = vals.clone()
    slots = torch.zeros(n, dtype=torch.float32, device=cuda_device)
    flags = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    st = srdit.ops.peer_ptrs([slots.data_ptr()])
    ft = srdit.ops.peer_ptrs([flags.data_ptr()])
    out = torch.full((n,), -7.0, device=cuda_device)
    L = srdit._lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    args = (ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(out.data_ptr()), n,
            srdit._lib.SRDIT_RED_SUM, ctypes.byref(st), ctypes.byref(ft), 0, 1, 2,
            ctypes.c_void_p(status.data_ptr()), stream)
    assert L.srdit_tp_allreduce(*args) == 0
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == srdit._lib.SRDIT_STATUS_TIMEOUT
    assert bool((out == -7.0).all())
    status.zero_()
    assert L.srdit_tp_allreduce(*args) == 0
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0 and int(flags[0].item()) == 2 * srdit._lib.SRDIT_AR_BLOCKS
    assert torch.equal(out, vals)


@pytest.mark.parametrize("f_cur,f_kv,bhw,rhw,anchor", [
    (1, 1, (8, 8), (0, 0), None),      # one KV tile per item: one group has none
    (3, 3, (8, 8), (0, 0), None),      # two tiles per item
    (3, 6, (4, 4), (1, 1), "frame"),   # many tiles, per-frame anchor tiles, window pairs
])
def test_winattn_split_kv_schedule_forced(srdit, cuda_device, f_cur, f_kv, bhw, rhw, anchor):
    """The split-KV schedule (two softmax groups on alternate KV tiles, each with
    its own O, combined at the item's end) forced onto plans the planner would
    run on the other schedule, including items whose single KV tile leaves one
    group without work; against the oracle and the other schedule."""
    h, w, n = 8, 16, 2
    L = h * w
    gen = torch.Generator().manual_seed(41 + f_cur + f_kv)
    q = torch.randn(f_cur * L, n, 128, generator=gen).to(torch.bfloat16)
    a_tok = f_cur * L if anchor else 0
    k = torch.randn(a_tok + f_kv * L, n, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(a_tok + f_kv * L, n, 128, generator=gen).to(torch.bfloat16)
    spec = obg.make_spec(f_cur, f_kv, h, w, block_t=3, block_hw=bhw, block_radius_hw=rhw,
                         streaming=f_kv > f_cur or anchor is not None)
    oplan = obg.build_plan(spec, anchor)
    ref = owa.run_plan(q, k, v, oplan, f_cur=f_cur, h=h, w=w)
    outs = []
    for split in (0, 1):
        plan = {"params": torch.as_tensor(oplan["params"]), "n_w": oplan["n_w"],
                "p_stride": oplan["p_stride"], "hr_base": oplan["hr_base"]}
        out = torch.empty_like(q, device=cuda_device)
        d = lambda t: t.to(cuda_device)  # noqa: E731
        srdit.attention.run_blockgrid_b200(d(q), d(k), d(v), out, plan=plan, f_cur=f_cur, h=h,
                                           w=w, n=n, d=128, anchor_mode=anchor)
        plan[("b200", out.device)][1].split_kv = split   # the launch's tiling record
        srdit.attention.run_blockgrid_b200(d(q), d(k), d(v), out, plan=plan, f_cur=f_cur, h=h,
                                           w=w, n=n, d=128, anchor_mode=anchor)
        torch.cuda.synchronize(cuda_device)
        _check_attn(out, ref)
        outs.append(out.float())
    assert onum.rel_fro(outs[1], outs[0]) < 5e-3
