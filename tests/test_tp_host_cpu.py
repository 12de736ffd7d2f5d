"""Tensor-parallel host orchestration on the CPU: two gloo ranks, no GPU.

The sharded forward (``TPSRDiT`` with library collectives) and the single-rank
forward (``SRDiT``) run with the CPU test double of the kernel launchers
(``tests/cpu_ops.py``). What this checks is the host side of tensor
parallelism: how each rank slices and quantises the weights (per-channel
scales over the full input width for row-parallel Linears), the sequence split
of the residual stream, and where each all-gather / reduce-scatter / all-reduce
sits. Two ranks must reproduce one rank's output (cosine >= 0.999; what
differs is the summation order and the bf16 rounding of each rank's partial).
"""
import datetime
import importlib
import multiprocessing as mp
import pathlib
import socket
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CFG = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, in_dim=16, out_dim=16, text_dim=64,
           text_len=16, block_hw=(2, 2), block_radius_hw=(1, 1))
GRID = (3, 4, 8)


def _run(model, torch, cfg, lat, ctx):
    """A cache-refresh forward, then a streaming forward that uses the
    per-context text cache (each rank's share of the cross K / V)."""
    f, h, w = GRID
    ring = model.new_cache(h * w)
    a = model.forward_chunk(lat[0], 0.0, ctx, cache=ring, update_cache=True)
    text = model.text_cache(ctx)
    b = model.forward_chunk(lat[1], 625.0, ctx, cache=ring, t_offset=f, text=text)
    model.check_status()
    return a.float(), b.float()


def _worker(rank, world, port, out_q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    try:
        torch.set_num_threads(2)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=120))
        importlib.import_module("dreamx-creator_b200")
        M = importlib.import_module("dreamx-creator_b200.model")
        T = importlib.import_module("dreamx-creator_b200.tp")
        from tests import cpu_ops

        class CpuTP(T.TPSRDiT):
            ops = cpu_ops
            require_cuda = False

        class CpuOne(M.SRDiT):
            ops = cpu_ops
            require_cuda = False

        cfg = M.SRDiTConfig(**CFG)
        f, h, w = GRID
        g = torch.Generator().manual_seed(5)
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
        lat = [torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
               for _ in range(2)]
        sd = M.SRDiT.seeded_state_dict(cfg, "cpu", 3)
        tp_out = _run(CpuTP(cfg, sd, "cpu", fused=False), torch, cfg, lat, ctx)
        res = None
        if rank == 0:
            ref = _run(CpuOne(cfg, sd, "cpu"), torch, cfg, lat, ctx)
            res = []
            for x, y in zip(tp_out, ref):
                x, y = x.double().reshape(-1), y.double().reshape(-1)
                res.append(float(torch.dot(x, y) / (x.norm() * y.norm())))
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback
        out_q.put((rank, None, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def test_tp2_gloo_matches_one_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, res, err = q.get(timeout=300)
            results[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errs = [e for _, e in results.values() if e]
    assert not errs, errs
    cos = results[0][0]
    assert min(cos) >= 0.999, cos


def _kv_only_worker(rank, world, port, out_q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    try:
        torch.set_num_threads(2)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=120))
        importlib.import_module("dreamx-creator_b200")
        M = importlib.import_module("dreamx-creator_b200.model")
        T = importlib.import_module("dreamx-creator_b200.tp")
        from tests import cpu_ops

        class CpuTP(T.TPSRDiT):
            ops = cpu_ops
            require_cuda = False

        cfg = M.SRDiTConfig(**CFG)
        f, h, w = GRID
        g = torch.Generator().manual_seed(7)
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
        lat = torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
        sd = M.SRDiT.seeded_state_dict(cfg, "cpu", 3)
        rings = []
        for kv_only in (False, True):
            model = CpuTP(cfg, sd, "cpu", fused=False)
            ring = model.new_cache(h * w)
            out = model.forward_chunk(lat, 0.0, ctx, cache=ring, update_cache=True,
                                      kv_only=kv_only)
            assert (out is None) == kv_only
            rings.append(ring)
        same = all(torch.equal(x, y) for x, y in zip(rings[0].k + rings[0].v,
                                                       rings[1].k + rings[1].v))
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, same, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback
        out_q.put((rank, None, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def test_tp2_refresh_kv_only_fills_the_same_ring():
    """Two gloo ranks: the kv_only refresh (last block stops after its K / V,
    no head, no final all-gather) leaves every rank's ring slice equal to the
    full refresh forward's."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_kv_only_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, same, err = q.get(timeout=300)
            results[rank] = (same, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errs = [e for _, e in results.values() if e]
    assert not errs, errs
    assert all(same for same, _ in results.values()), results


def test_single_rank_model_refuses_cpu():
    """Without the test double and without CUDA the model does not build."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    M = importlib.import_module("dreamx-creator_b200.model")
    srdit = importlib.import_module("dreamx-creator_b200")
    cfg = M.SRDiTConfig(**CFG)
    with pytest.raises(srdit._lib.SrditError):
        M.SRDiT(cfg, M.SRDiT.seeded_state_dict(cfg, "cpu", 3), "cpu")


def _harvest_worker(rank, world, port, out_q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    try:
        torch.set_num_threads(2)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=120))
        importlib.import_module("dreamx-creator_b200")
        M = importlib.import_module("dreamx-creator_b200.model")
        T = importlib.import_module("dreamx-creator_b200.tp")
        from tests import cpu_ops

        class CpuTP(T.TPSRDiT):
            ops = cpu_ops
            require_cuda = False

        cfg = M.SRDiTConfig(**CFG)
        f, h, w = GRID
        g = torch.Generator().manual_seed(21)
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
        lq = torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
        sd = M.SRDiT.seeded_state_dict(cfg, "cpu", 3)
        model = CpuTP(cfg, sd, "cpu", fused=False)
        _, kv = model.forward_chunk(lq, 0.0, ctx, cache=None, t_offset=2, return_kv=True,
                                    independent_frames=True)
        per = [model.forward_chunk(lq[:, j:j + 1], 0.0, ctx, cache=None, t_offset=2 + j,
                                   return_kv=True)[1] for j in range(f)]
        worst = 1.0
        for li, (k, v) in enumerate(kv):
            for got, ref in ((k, torch.cat([p[li][0] for p in per])),
                             (v, torch.cat([p[li][1] for p in per]))):
                x, y = got.double().reshape(-1), ref.double().reshape(-1)
                worst = min(worst, float(torch.dot(x, y) / (x.norm() * y.norm())))
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, worst, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback
        out_q.put((rank, None, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def test_tp2_batched_harvest_matches_per_frame_forwards():
    """Two gloo ranks: each rank's share of the anchor harvest run as one
    forward over independent frames equals its share from one 1-frame forward
    per frame (cosine >= 0.9999; the double's float matmul may block rows
    differently for 1 and 3 frames)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_harvest_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, worst, err = q.get(timeout=300)
            results[rank] = (worst, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errs = [e for _, e in results.values() if e]
    assert not errs, errs
    assert min(w for w, _ in results.values()) >= 0.9999, results


def _anchor_worker(rank, world, port, out_q):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    try:
        torch.set_num_threads(2)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=120))
        importlib.import_module("dreamx-creator_b200")
        M = importlib.import_module("dreamx-creator_b200.model")
        T = importlib.import_module("dreamx-creator_b200.tp")
        P = importlib.import_module("dreamx-creator_b200.pipeline")
        from tests import cpu_ops

        class CpuTP(T.TPSRDiT):
            ops = cpu_ops
            require_cuda = False

        class CpuOne(M.SRDiT):
            ops = cpu_ops
            require_cuda = False

        cfg = M.SRDiTConfig(**CFG)
        f, h, w = GRID
        g = torch.Generator().manual_seed(31)
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
        lq = torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
        x = torch.randn(cfg.in_dim, f, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
        sd = M.SRDiT.seeded_state_dict(cfg, "cpu", 3)

        def run(model):
            stream = P.RefinerStream(model, ctx)
            stream._ensure_text()
            anchor = stream.harvest_anchor(lq)
            return model.forward_chunk(x, 625.0, ctx, cache=None, anchor_kv=anchor,
                                       text=stream.text).float()

        tp_out = run(CpuTP(cfg, sd, "cpu", fused=False))
        cos = None
        if rank == 0:
            ref = run(CpuOne(cfg, sd, "cpu"))
            a, b = tp_out.double().reshape(-1), ref.double().reshape(-1)
            cos = float(torch.dot(a, b) / (a.norm() * b.norm()))
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, cos, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback
        out_q.put((rank, None, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def test_tp2_anchor_harvest_and_frame_anchor_match_one_rank():
    """Two gloo ranks: the LQ-anchor path (each rank harvests its heads' share
    of the anchor in one forward, then a frame-aligned anchored denoise)
    reproduces one rank's output (cosine >= 0.999)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_anchor_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, cos, err = q.get(timeout=300)
            results[rank] = (cos, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errs = [e for _, e in results.values() if e]
    assert not errs, errs
    assert results[0][0] >= 0.999, results
