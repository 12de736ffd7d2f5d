"""BASELINE config 3 at full width: one 2K chunk of the SR-DiT 5B forward.

dim 3072, 24 heads x 128, FFN 14336, 48-channel latent of 3 frames at 72 x 128
(36 x 64 tokens per frame, 6912 tokens), a 3-frame KV-cache prefix (the chunk
attends f_kv = 6 frames), a 512-token N(0,1) 4096-d text context, t = 625,
temporal offset 3, fp8 Linears, seeded random weights -- with 2 of the 30
blocks, so that the CPU oracle (video_refiner/wan/modules/sr_dit/models.py:
1877-2002 restated in oracle/model.py, fp64-accumulated fp8 products) finishes
in about a minute. Three cases: BASELINE's literal 3x8x8 windows, the shipped
4x4 radius-3 windows, and the shipped default denoise with a frame-aligned LQ
anchor. Each compares every block's output hidden state, the chunk's roped K /
raw V written into the cache, and the refined prediction with the oracle:
cosine >= 0.999 (the full-latent tolerance).
"""
import dataclasses
import importlib
import os
from types import SimpleNamespace

import pytest
import torch

from oracle import model as omodel
from oracle import numerics as onum

pytestmark = pytest.mark.gpu

LAYERS = 2
L = 36 * 64
bf16 = torch.bfloat16


@pytest.fixture(scope="module")
def c3(srdit, cuda_device):
    torch.set_num_threads(os.cpu_count() or 1)
    M = importlib.import_module("dreamx-creator_b200.model")
    cfg = M.SRDiTConfig(num_layers=LAYERS)
    lazy = M.SRDiT.seeded_state_dict(cfg, cuda_device, seed=0)
    sd = {n: lazy[n].cpu() for n in M.SRDiT.param_shapes(cfg)}
    model = M.SRDiT(dataclasses.replace(cfg), {n: v.to(cuda_device) for n, v in sd.items()},
                    cuda_device)
    g = torch.Generator().manual_seed(2024)
    lat = torch.randn(48, 3, 72, 128, generator=g).to(bf16)
    ctx = torch.randn(512, 4096, generator=g).to(bf16)
    rnd = lambda: torch.randn(3 * L, 3072, generator=g).to(bf16)  # noqa: E731
    prefix = [(rnd(), rnd()) for _ in range(LAYERS)]
    anchor = [(rnd(), rnd()) for _ in range(LAYERS)]
    return SimpleNamespace(cfg=cfg, sd=sd, model=model, lat=lat, ctx=ctx, prefix=prefix,
                           anchor=anchor, fp8c=[dict() for _ in range(LAYERS)], dev=cuda_device)


@pytest.mark.parametrize("geometry,anchored", [(((8, 8), (0, 0)), False),
                                               (((4, 4), (3, 3)), False),
                                               (((4, 4), (3, 3)), True)],
                         ids=["8x8r0", "4x4r3", "4x4r3_frame_anchor"])
def test_config3_full_width_chunk_matches_oracle(c3, geometry, anchored):
    bhw, rhw = geometry
    model, dev = c3.model, c3.dev
    model.cfg.block_hw, model.cfg.block_radius_hw = bhw, rhw
    ring = model.new_cache(L)
    for li, (k, v) in enumerate(c3.prefix):
        ring.k[li][:3 * L].copy_(k.to(dev))
        ring.v[li][:3 * L].copy_(v.to(dev))
    ring.start, ring.frames = 0, 3
    anchor_dev = [(k.to(dev), v.to(dev)) for k, v in c3.anchor] if anchored else None
    outs = []
    y = model.forward_chunk(c3.lat.to(dev), 625.0, c3.ctx.to(dev), cache=ring, t_offset=3,
                            anchor_kv=anchor_dev, anchor_align="frame", block_outputs=outs)
    torch.cuda.synchronize(dev)
    model.check_status()
    ocfg = dataclasses.replace(c3.cfg, block_hw=bhw, block_radius_hw=rhw)
    heads = lambda t: t.view(-1, 24, 128)  # noqa: E731
    ref_outs = []
    ref, caches = omodel.forward_chunk(
        c3.sd, ocfg, c3.lat, 625.0, c3.ctx,
        caches=[(heads(k), heads(v)) for k, v in c3.prefix], t_offset=3, kv_len=9,
        fp8caches=c3.fp8c,
        anchor=[(heads(k), heads(v)) for k, v in c3.anchor] if anchored else None,
        anchor_align="frame", block_outputs=ref_outs)
    assert len(outs) == len(ref_outs) == LAYERS
    for li in range(LAYERS):
        c = onum.cosine(outs[li].float().cpu(), ref_outs[li].float())
        assert c >= 0.999, ("block output", li, c)
        # this chunk's roped K and raw V in ring slots 3..5 vs the oracle cache tail
        for got, want in ((ring.k[li][3 * L:6 * L], caches[li][0][-3 * L:]),
                          (ring.v[li][3 * L:6 * L], caches[li][1][-3 * L:])):
            c = onum.cosine(got.float().cpu(), want.reshape(3 * L, 3072).float())
            assert c >= 0.999, ("cache", li, c)
    c = onum.cosine(y.float().cpu(), ref.float())
    assert c >= 0.999, ("prediction", c)
