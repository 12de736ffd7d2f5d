"""The spatial (window-strip) partition on two gloo ranks with the CPU test
double of the kernel launchers: each rank refines half of the token columns,
and the gathered prediction must match the one-rank forward over the whole
grid -- chunks over a refreshed cache (RoPE at the strip's true width
positions, the strip's own ring) and an anchored chunk (the harvest on each
strip)."""
import datetime
import importlib
import pathlib
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = pathlib.Path(__file__).resolve().parents[1]
CFG = dict(dim=256, ffn_dim=512, num_heads=2, num_layers=2, in_dim=16, out_dim=16, text_dim=64,
           text_len=16, block_hw=(2, 4), block_radius_hw=(1, 0))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stream_outputs(P, model, torch, cfg):
    g = torch.Generator().manual_seed(5)
    ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(torch.bfloat16)
    chunks = [torch.randn(cfg.in_dim, 3, 8, 32, generator=g).to(torch.bfloat16)
              for _ in range(2)]
    lq = torch.randn(cfg.in_dim, 3, 8, 32, generator=g).to(torch.bfloat16)
    stream = P.RefinerStream(model, ctx)
    res = [stream.step(c).float() for c in chunks]
    res.append(stream.step(chunks[0], lq_chunk=lq).float())
    stream.check_status()
    return res


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
        S = importlib.import_module("dreamx-creator_b200.spatial")
        P = importlib.import_module("dreamx-creator_b200.pipeline")
        from tests import cpu_ops

        class CpuSpatial(S.SpatialSRDiT):
            ops = cpu_ops
            require_cuda = False

        class CpuOne(M.SRDiT):
            ops = cpu_ops
            require_cuda = False

        cfg = M.SRDiTConfig(**CFG)
        sd = M.SRDiT.seeded_state_dict(cfg, "cpu", 3)
        got = _stream_outputs(P, CpuSpatial(cfg, sd, "cpu"), torch, cfg)
        res = None
        if rank == 0:
            ref = _stream_outputs(P, CpuOne(cfg, sd, "cpu"), torch, cfg)
            res = []
            for x, y in zip(got, ref):
                assert x.shape == y.shape, (x.shape, y.shape)
                x, y = x.double().reshape(-1), y.double().reshape(-1)
                res.append(float(torch.dot(x, y) / (x.norm() * y.norm())))
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback
        out_q.put((rank, None, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-1500:]}"))


def test_two_strips_match_one_rank():
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
    assert len(cos) == 3 and min(cos) > 0.9999, cos


def test_radius_along_w_is_refused(monkeypatch):
    import torch.distributed as dist
    importlib.import_module("dreamx-creator_b200")
    S = importlib.import_module("dreamx-creator_b200.spatial")
    M = importlib.import_module("dreamx-creator_b200.model")
    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(dist, "get_world_size", lambda g=None: 2)
    monkeypatch.setattr(dist, "get_rank", lambda g=None: 0)
    cfg = M.SRDiTConfig(**{**CFG, "block_radius_hw": (1, 1)})
    with pytest.raises(M._lib.SrditError, match="radius 0 along w"):
        S.SpatialSRDiT(cfg, {}, "cpu")
