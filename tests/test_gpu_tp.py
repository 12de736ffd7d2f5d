"""Tensor-parallel forward (TP=2) against the single-GPU forward.

Two spawned ranks run the sharded model on one clip -- with the collectives
fused into the kernels over peer memory (the all-gather stored by the LN
kernel itself, or pushed by the copy engines), and with NCCL collectives -- a
cache-refresh forward,
then a streaming forward over the ring it filled. Rank 0 also runs the same
seeded weights unsharded (``SRDiT``, which the other GPU tests pin to the CPU
oracle) and compares both outputs. What differs between the two is only the
fp32 summation order of the full-row statistics and the bf16 rounding of each
rank's partial product before the reduce-scatter; tolerance: cosine >= 0.999
(the model-level bar of the refiner's numerics contract).
"""
import importlib
import multiprocessing as mp
import os
import pathlib
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = pathlib.Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg_kw, grid, fused, out_q, graphs=False):
    import datetime
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        importlib.import_module("dreamx-creator_b200")
        M = importlib.import_module("dreamx-creator_b200.model")
        T = importlib.import_module("dreamx-creator_b200.tp")
        cfg = M.SRDiTConfig(**cfg_kw)
        dev = torch.device("cuda", rank)
        f, h, w = grid
        g = torch.Generator().manual_seed(5)
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16).to(dev)
        lat = [torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16).to(dev)
               for _ in range(2)]

        def run(model):
            ring = model.new_cache(h * w, grid_hw=(h, w))
            a = model.forward_chunk(lat[0], 0.0, ctx, cache=ring, update_cache=True)
            b = model.forward_chunk(lat[1], 625.0, ctx, cache=ring, t_offset=f)
            torch.cuda.synchronize()
            model.check_status()
            return a.float().cpu(), b.float().cpu()

        if graphs:
            # the refiner loop with captured steps: 5 chunks over a 6-slot ring
            Pm = importlib.import_module("dreamx-creator_b200.pipeline")
            lat5 = [torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
                    .to(dev) for _ in range(5)]

            def run(model, graphed=True):  # noqa: F811
                stream = Pm.RefinerStream(model, ctx, graphs=graphed)
                outs = [stream.step(x).float().cpu() for x in lat5]
                # an anchored step: the LR frames' harvest, then the anchor's columns
                outs.append(stream.step(lat5[0], lq_chunk=lat5[1]).float().cpu())
                torch.cuda.synchronize()
                model.check_status()
                return outs
        if str(fused).startswith("spatial"):   # the window-strip partition instead of TP
            S = importlib.import_module("dreamx-creator_b200.spatial")
            halo = fused.split(":")[1] if ":" in fused else "peer"
            tp_model = S.SpatialSRDiT.random_init(cfg, dev, seed=3, halo=halo)
        elif fused == "ce":   # peer-fused, all-gather pushed by the copy engines
            tp_model = T.TPSRDiT.random_init(cfg, dev, seed=3, comm=T.PeerComm(push="ce"))
        else:
            tp_model = T.TPSRDiT.random_init(cfg, dev, seed=3, fused=fused)
        tp_out = run(tp_model)
        res = None
        if rank == 0:
            ref_model = M.SRDiT.random_init(cfg, dev, seed=3)
            ref_out = run(ref_model, False) if graphs else run(ref_model)
            cos = []
            for x, y in zip(tp_out, ref_out):
                x, y = x.double().reshape(-1), y.double().reshape(-1)
                cos.append(float(torch.dot(x, y) / (x.norm() * y.norm())))
            res = cos
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, None, f"{type(e).__name__}: {e}"))


def _run_tp(world, cfg_kw, grid, fused, graphs=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_kw, grid, fused, q, graphs))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, res, err = q.get(timeout=600)
            results[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errs = [e for _, e in results.values() if e]
    assert not errs, errs
    return results[0][0]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [True, "ce", False], ids=["peer-fused", "peer-ce", "nccl"])
@pytest.mark.parametrize("cfg_kw,grid", [
    (dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, in_dim=16, out_dim=16, text_dim=64,
          text_len=16, block_hw=(2, 2), block_radius_hw=(1, 1)), (3, 8, 16)),
    (dict(num_layers=2, block_hw=(8, 8), block_radius_hw=(0, 0)), (3, 36, 64)),
], ids=["small", "2K-2layers"])
def test_tp2_matches_single_gpu(cfg_kw, grid, fused):
    cos = _run_tp(2, cfg_kw, grid, fused)
    assert min(cos) >= 0.999, cos


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_graph_replay_matches_single_gpu():
    """The fused TP forward captured in CUDA graphs (peer counters reset per
    forward, copy-engine pushes and NCCL inside the graph) against the eager
    single-GPU refiner loop over 5 chunks."""
    cfg_kw = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, in_dim=16, out_dim=16,
                  text_dim=64, text_len=16, block_hw=(2, 2), block_radius_hw=(1, 1), kv_len=3)
    cos = _run_tp(2, cfg_kw, (3, 8, 16), True, graphs=True)
    assert min(cos) >= 0.999, cos


_SMALL = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, in_dim=16, out_dim=16,
              text_dim=64, text_len=16, block_hw=(2, 4), kv_len=3)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graphs"])
@pytest.mark.parametrize("cfg_kw,grid,halo", [
    (dict(_SMALL, block_radius_hw=(1, 0)), (3, 8, 16), "peer"),
    (dict(num_layers=2, block_hw=(8, 8), block_radius_hw=(0, 0)), (3, 36, 64), "peer"),
    (dict(_SMALL, block_radius_hw=(1, 1)), (3, 8, 16), "peer"),
    (dict(_SMALL, block_radius_hw=(1, 1)), (3, 8, 16), "collective"),
    (dict(num_layers=2, block_hw=(4, 4), block_radius_hw=(3, 3)), (3, 36, 64), "peer"),
], ids=["small", "2K-8x8r0-2layers", "small-halo-peer", "small-halo-nccl",
        "2K-4x4r3-2layers-halo-peer"])
def test_spatial2_matches_single_gpu(cfg_kw, grid, halo, graphs):
    """The window-strip partition on two GPUs (each refines half of the token
    columns with the full model, one all-gather per forward; eager and in
    captured CUDA graphs, with an anchored step) against the single-GPU
    forward. With radius > 0 along w the strips' K/V halo columns cross GPUs
    every block: stored into the neighbour's ring by the ring-write kernel
    ("peer") or sent with NCCL point-to-point calls ("nccl")."""
    cos = _run_tp(2, cfg_kw, grid, "spatial:" + halo, graphs=graphs)
    assert min(cos) >= 0.999, cos
