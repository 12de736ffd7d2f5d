"""The kernels at the shapes a tensor-parallel rank runs them (one GPU).

At TP = 2 / 4 / 8 a rank holds 12 / 6 / 3 heads, 1536 / 768 / 384 of the 3072
features and 7168 / 3584 / 1792 FFN columns, and its full-row statistics (the
RMSNorm sum of squares, the per-token fp8 amax) come from an all-reduce. These
tests run each kernel on such a slice with the full-row statistic passed in and
compare with the oracle applied to the full row, then sliced.
"""
import numpy as np
import pytest
import torch

from oracle import numerics as onum
from oracle import winattn as owa

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_rms_rope_slice_with_full_row_sumsq(srdit, cuda_device, world):
    f, h, w, D = 2, 5, 8, 3072
    Dl = D // world
    M = f * h * w
    g = torch.Generator().manual_seed(31 + world)
    x = torch.randn(M, D, generator=g).to(torch.bfloat16)
    wt = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    freqs = onum.rope_freqs()
    cos, sin = onum.rope_tables(freqs)
    ref = onum.rope_apply(onum.rms_norm(x, wt).view(M, 24, 128), (f, h, w), freqs, 3).view(M, D)
    ss_full = x.float().pow(2).sum(-1)
    for r in range(world):
        sl = slice(r * Dl, (r + 1) * Dl)
        dst = torch.empty(M, Dl, dtype=torch.bfloat16, device=cuda_device)
        srdit.ops.rms_rope(x[:, sl].contiguous().to(cuda_device), wt[sl].contiguous().to(cuda_device),
                           1e-6, dst, frame_tokens=h * w, cos=cos.to(cuda_device),
                           sin=sin.to(cuda_device), grid_h=h, grid_w=w, t_offset=3,
                           ss=ss_full.to(cuda_device), norm_width=D)
        assert onum.rel_fro(dst.cpu().float(), ref[:, sl].float()) < 1e-3


@pytest.mark.parametrize("K", [384, 768, 1792, 3584])
def test_quant_slice_with_global_amax(srdit, cuda_device, K):
    M = 200
    g = torch.Generator().manual_seed(K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    amax = x.float().abs().amax(-1) * (1 + torch.rand(M, generator=g))  # the full row's
    q, s = srdit.ops.quant_rowwise(x.to(cuda_device), amax=amax.to(cuda_device))
    s_ref = (amax / onum.FP8_MAX).clamp_min(1e-12)
    q_ref = (x.float() / s_ref[:, None]).clamp(-onum.FP8_MAX, onum.FP8_MAX) \
        .to(torch.float8_e4m3fn)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref.numpy())
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(),
                                  q_ref.view(torch.uint8).numpy())
    # without amax: the row's own
    q2, s2 = srdit.ops.quant_rowwise(x.to(cuda_device))
    qo, so = onum.quantize_rowwise(x)
    np.testing.assert_array_equal(q2.view(torch.uint8).cpu().numpy(),
                                  qo.view(torch.uint8).numpy())


@pytest.mark.parametrize("M,N,K", [(864, 3072, 384), (1728, 1152, 3072), (6912, 3072, 1792)])
def test_fp8_gemm_rank_shapes(srdit, cuda_device, M, N, K):
    g = torch.Generator().manual_seed(M + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    aq, as_ = onum.quantize_rowwise(a)
    wq, ws = onum.fp8_linear_weights(w)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    out = srdit.ops.fp8_gemm(d(aq), d(as_.reshape(-1).contiguous()), d(wq), d(ws))
    ref = onum.fp8_linear(a, wq, ws, None)
    assert onum.rel_fro(out.cpu().float(), ref.float()) < 1e-3


def test_winattn_three_heads(srdit, cuda_device):
    """The TP = 8 rank's 3 heads, 2K 8x8 windows, a 3-frame cache."""
    n, f_cur, f_kv, h, w = 3, 3, 6, 36, 64
    L = h * w
    spec = srdit.blockgrid.make_spec(f_cur=f_cur, f_kv=f_kv, h=h, w=w, block_t=3,
                                     block_hw=(8, 8), block_radius_hw=(0, 0), streaming=True)
    plan = srdit.attention.cached_plan(spec)
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(f_cur * L, n, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(f_kv * L, n, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(f_kv * L, n, 128, generator=gen).to(torch.bfloat16)
    out = torch.empty_like(q, device=cuda_device)
    srdit.attention.run_blockgrid_b200(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                       out, plan=plan, f_cur=f_cur, h=h, w=w, n=n, d=128)
    ref = owa.run_plan(q, k, v, {"params": plan["params"].numpy(), "hr_base": 0,
                                 "p_stride": plan["p_stride"]}, f_cur=f_cur, h=h, w=w)
    got = out.float().cpu().double()
    assert (got - ref.double()).abs().max().item() <= 2e-2
    assert onum.rel_fro(got, ref.double()) <= 5e-3


@pytest.mark.parametrize("gated", [True, False])
def test_residual_sum_of_parts(srdit, cuda_device, gated):
    S, M, N = 8, 96, 3072
    g = torch.Generator().manual_seed(8)
    parts = (torch.randn(S, M, N, generator=g) * 0.1).to(torch.bfloat16)
    x = torch.randn(M, N, generator=g).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    gate = torch.randn(N, generator=g) * 0.5 if gated else None
    xd = x.to(cuda_device)
    srdit.ops.residual(xd, parts.to(cuda_device), bias=bias.to(cuda_device),
                       gate=gate.to(cuda_device) if gated else None)
    y = parts.float().sum(0) + bias.float()
    y = y.to(torch.bfloat16).float()
    ref = (x.float() + y * gate) if gated else (x.float() + y)
    ref = ref.to(torch.bfloat16)
    diff = (xd.cpu().float() - ref.float()).abs()
    # the 8-way fp32 sum is taken in another order than torch's: rare 1-ulp ties
    assert (diff == 0).float().mean() > 0.99
    assert onum.rel_fro(xd.cpu().float(), ref.float()) < 1e-3


@pytest.mark.parametrize("K", [384, 1536])
def test_row_reduce(srdit, cuda_device, K):
    M = 300
    g = torch.Generator().manual_seed(K + 1)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    ss = srdit.ops.row_reduce(x.to(cuda_device), "sumsq").cpu()
    am = srdit.ops.row_reduce(x.to(cuda_device), "absmax").cpu()
    np.testing.assert_allclose(ss.numpy(), x.float().pow(2).sum(-1).numpy(), rtol=1e-5)
    np.testing.assert_array_equal(am.numpy(), x.float().abs().amax(-1).numpy())


@pytest.mark.parametrize("world,rank,M,affine", [(1, 0, 1000, False), (2, 1, 3456, False),
                                                 (8, 5, 864, False), (8, 0, 1001, True),
                                                 (4, 3, 7, True), (2, 0, 6913, False)])
def test_ln_mod_quant_allgather_local_ranks(srdit, cuda_device, world, rank, M, affine):
    """The LN-modulate-quantise all-gather with every rank's gather buffer on this
    GPU: the rank's rows (a block of M rows at row rank * M) must land in all
    `world` buffers byte-equal to the single-GPU kernel's, the row scales too, and
    every other rank's flag word must count the launch once (none for the rank
    itself). At 3456 and 6913 rows each CTA of the persistent grid runs several
    row groups."""
    K = 3072
    g = torch.Generator().manual_seed(world * 100 + M)
    x = (torch.randn(M, K, generator=g) * 2 + 0.3).to(torch.bfloat16)
    shift = scale = w = b = None
    if affine:
        w = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
        b = (0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    else:
        shift, scale = 0.1 * torch.randn(K, generator=g), 0.1 * torch.randn(K, generator=g)
    dev = lambda t: None if t is None else t.to(cuda_device)  # noqa: E731
    rows = world * M
    q = [torch.zeros(rows, K, dtype=torch.uint8, device=cuda_device) for _ in range(world)]
    s = [torch.zeros(rows, dtype=torch.float32, device=cuda_device) for _ in range(world)]
    flags = [torch.zeros(8, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    done = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    qt, st, ft = srdit._lib.PeerPtrs(), srdit._lib.PeerPtrs(), srdit._lib.PeerPtrs()
    for d in range(world):
        qt.p[d] = q[d][rank * M:].data_ptr()
        st.p[d] = s[d][rank * M:].data_ptr()
        ft.p[d] = flags[d].data_ptr()
    srdit.ops.ln_mod_quant_tp(dev(x), 1e-6, ln_weight=dev(w), ln_bias=dev(b), shift=dev(shift),
                              scale=dev(scale), q_rows=qt, s_rows=st, flags=ft, done=done,
                              rank=rank, world=world, ldq=K)
    torch.cuda.synchronize()
    # the single-GPU kernel runs the same arithmetic: its bytes are the reference
    q1, s1 = srdit.ops.ln_mod_quant(dev(x), 1e-6, ln_weight=dev(w), ln_bias=dev(b),
                                    shift=dev(shift), scale=dev(scale))
    blk = slice(rank * M, (rank + 1) * M)
    for d in range(world):
        assert torch.equal(q[d][blk], q1.view(torch.uint8)), d
        assert torch.equal(s[d][blk], s1), d
        # nothing outside the rank's block is written
        assert int(q[d].view(-1).count_nonzero()) == int(q[d][blk].view(-1).count_nonzero())
        want = [0] * 8
        if d != rank:
            want[rank] = 1
        assert flags[d].cpu().tolist() == want, (d, flags[d])
    assert int(done.item()) == 0
    # and the oracle: the LN statistics are reduced in another order than torch's
    # CPU kernel, so at thousands of rows a bf16 tie can move a row's amax by one
    # ulp and rescale that row's bytes (measured up to 4.3e-4 on these inputs)
    n = onum.layer_norm(x, 1e-6, w, b)
    if not affine:
        n = (n.float() * (1 + scale) + shift).to(torch.bfloat16)
    qo, so = onum.quantize_rowwise(n)
    assert onum.rel_fro(q1.float().cpu() * s1.cpu()[:, None], qo.float() * so) < 1e-3
