"""The LQ-anchor harvest as one forward, on the CPU test double.

The reference harvests the anchor as one generator forward over the LR chunk's
frames as B = f independent 1-frame samples (causal_inference.py:456-460).
``forward_chunk(..., independent_frames=True)`` runs those samples side by
side in one chunk: the self-attention plan is the 1-frame plan repeated per
frame (frame j attends to frame j only), and frame j takes temporal position
t_offset + j. Its per-layer K / V must equal those of one 1-frame forward per
frame; everything else in the block is per token.
"""
import importlib

import pytest
import torch

from tests import cpu_ops

CFG = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, in_dim=16, out_dim=16, text_dim=64,
           text_len=16, block_hw=(2, 2), block_radius_hw=(1, 1))


def _model():
    M = importlib.import_module("dreamx-creator_b200.model")

    class CpuOne(M.SRDiT):
        ops = cpu_ops
        require_cuda = False

    cfg = M.SRDiTConfig(**CFG)
    return M, cfg, CpuOne(cfg, M.SRDiT.seeded_state_dict(cfg, "cpu", 11), "cpu")


def test_frames_plan_rows_are_the_one_frame_rows_per_frame():
    importlib.import_module("dreamx-creator_b200")
    A = importlib.import_module("dreamx-creator_b200.attention")
    B = importlib.import_module("dreamx-creator_b200.blockgrid")
    spec1 = B.make_spec(f_cur=1, f_kv=1, h=4, w=8, block_t=3, block_hw=(2, 2),
                        block_radius_hw=(1, 1))
    one, stride, _ = B.plan_rows(spec1, None)
    plan = A.frames_plan(spec1, 3)
    rows = plan["params"]
    assert plan["p_stride"] == stride and rows.shape[0] == 3 * one.shape[0]
    for j in range(3):
        blk = rows[j * one.shape[0]:(j + 1) * one.shape[0]]
        assert torch.equal(blk[:, 0], one[:, 0] + j) and torch.equal(blk[:, 6], one[:, 6] + j)
        assert torch.equal(blk[:, 1:6], one[:, 1:6]) and torch.equal(blk[:, 7:], one[:, 7:])
    # query frame j sees KV frame j only
    assert torch.equal(rows[:, 0], rows[:, 6]) and bool((rows[:, 1] == 1).all())
    assert bool((rows[:, 7] == 1).all())
    with pytest.raises(ValueError):
        A.frames_plan(B.make_spec(f_cur=3, f_kv=3, h=4, w=8, block_t=3, block_hw=(2, 2),
                                  block_radius_hw=(1, 1)), 3)


def test_batched_harvest_equals_per_frame_forwards():
    torch.manual_seed(0)
    M, cfg, model = _model()
    g = torch.Generator().manual_seed(12)
    ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
    lq = torch.randn(cfg.in_dim, 3, 8, 16, generator=g).to(torch.bfloat16)
    _, kv = model.forward_chunk(lq, 0.0, ctx, cache=None, t_offset=4, return_kv=True,
                                independent_frames=True)
    per = [model.forward_chunk(lq[:, j:j + 1], 0.0, ctx, cache=None, t_offset=4 + j,
                               return_kv=True)[1] for j in range(3)]
    assert len(kv) == cfg.num_layers
    for li, (k, v) in enumerate(kv):
        rk = torch.cat([p[li][0] for p in per])
        rv = torch.cat([p[li][1] for p in per])
        assert k.shape == rk.shape and v.shape == rv.shape
        # the double's float matmul may block rows differently for 1 and 3 frames
        torch.testing.assert_close(k.float(), rk.float(), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(v.float(), rv.float(), rtol=2e-2, atol=2e-2)
        assert (k.view(torch.int16) == rk.view(torch.int16)).float().mean() > 0.99
    model.check_status()


def test_independent_frames_refuses_a_cache_or_an_anchor():
    M, cfg, model = _model()
    g = torch.Generator().manual_seed(13)
    ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
    lq = torch.randn(cfg.in_dim, 3, 8, 16, generator=g).to(torch.bfloat16)
    ring = model.new_cache(4 * 8)
    model.forward_chunk(lq, 0.0, ctx, cache=ring, update_cache=True)
    with pytest.raises(M._lib.SrditError):
        model.forward_chunk(lq, 0.0, ctx, cache=ring, t_offset=3, independent_frames=True)


def test_prefetched_harvest_gives_the_serial_stream():
    """RefinerStream.step(..., next_lq_chunk=...) harvests the next chunk's anchor
    ahead (a side stream on the GPU; at once on this CPU double) with its own
    scratch; three anchored chunks must come out exactly as with the harvest
    done inside each step."""
    M, cfg, model = _model()
    P = importlib.import_module("dreamx-creator_b200.pipeline")
    g = torch.Generator().manual_seed(14)
    ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
    noisy = [torch.randn(cfg.in_dim, 3, 8, 16, generator=g).to(torch.bfloat16) for _ in range(3)]
    lq = [torch.randn(cfg.in_dim, 3, 8, 16, generator=g).to(torch.bfloat16) for _ in range(3)]
    outs = {}
    for prefetch in (False, True):
        stream = P.RefinerStream(model, ctx)
        res = []
        for i in range(3):
            nxt = lq[i + 1] if prefetch and i + 1 < 3 else None
            res.append(stream.step(noisy[i], lq_chunk=lq[i], next_lq_chunk=nxt).clone())
            if prefetch and nxt is not None:
                assert stream._pending is not None and stream._pending[0] == 3 * (i + 1)
        stream.check_status()
        outs[prefetch] = res
    for a, b in zip(outs[False], outs[True]):
        assert torch.equal(a, b)


def test_refine_clip_is_the_chunk_loop():
    """pipeline.refine_clip over a 2-chunk clip (anchors from the LQ latent,
    the second harvested ahead) equals stepping the chunks one by one."""
    M, cfg, model = _model()
    P = importlib.import_module("dreamx-creator_b200.pipeline")
    g = torch.Generator().manual_seed(21)
    ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
    lq = torch.randn(cfg.in_dim, 6, 8, 16, generator=g).to(torch.bfloat16)
    noise = torch.randn(cfg.in_dim, 6, 8, 16, generator=g).to(torch.bfloat16)
    noisy = P.sr_noise(lq, noise, 0.625)
    assert torch.equal(noisy, (0.375 * lq.float() + 0.625 * noise.float()).to(torch.bfloat16))
    got = P.refine_clip(P.RefinerStream(model, ctx), noisy, lq=lq)
    s = P.RefinerStream(model, ctx)
    ref = torch.cat([s.step(noisy[:, i:i + 3], lq_chunk=lq[:, i:i + 3]) for i in (0, 3)], 1)
    assert got.shape == noisy.shape and torch.equal(got, ref)
    with pytest.raises(ValueError):
        P.refine_clip(P.RefinerStream(model, ctx), noisy[:, :4])
