"""The spatial (window-strip) partition on two gloo ranks with the CPU test
double of the kernel launchers: each rank refines half of the token columns,
and the gathered prediction must match the one-rank forward over the whole
grid -- chunks over a refreshed cache (RoPE at the strip's true width
positions, the strip's own ring) and an anchored chunk (the harvest on each
strip). With windows that see neighbouring columns (radius 1 along w) the
strips exchange their K/V halo columns every block (torch.distributed
point-to-point over gloo: the "collective" halo)."""
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


def _worker(rank, world, port, out_q, radius_w):
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

        cfg = M.SRDiTConfig(**{**CFG, "block_radius_hw": (1, radius_w)})
        sd = M.SRDiT.seeded_state_dict(cfg, "cpu", 3)
        got = _stream_outputs(P, CpuSpatial(cfg, sd, "cpu", halo="collective"), torch, cfg)
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


@pytest.mark.parametrize("radius_w", [0, 1], ids=["radius0", "halo"])
def test_two_strips_match_one_rank(radius_w):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, radius_w)) for r in range(2)]
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


def test_strips_narrower_than_the_halo_are_refused():
    """The halo comes from the adjacent strips only: a strip must be at least
    radius_w x block_w columns wide."""
    importlib.import_module("dreamx-creator_b200")
    S = importlib.import_module("dreamx-creator_b200.spatial")
    M = importlib.import_module("dreamx-creator_b200.model")
    m = object.__new__(S.SpatialSRDiT)
    m.cfg = M.SRDiTConfig(**{**CFG, "block_radius_hw": (1, 3)})
    m.world, m.rank, m.R = 2, 0, 3 * 4
    assert m.strip(32) == (0, 16) and m._ext_of(0, 32) == (0, 28)
    assert m._ext_of(1, 32) == (4, 32)
    with pytest.raises(M._lib.SrditError, match="narrower than the 12-column"):
        m.strip(16)


def test_strip_rows_keep_each_windows_keys():
    """A strip's rows (blockgrid.strip_rows) address, in the strip's K/V frame
    coordinates, exactly the full plan's query and key columns of its windows."""
    import torch
    importlib.import_module("dreamx-creator_b200")
    bg = importlib.import_module("dreamx-creator_b200.blockgrid")
    for mode in (None, "chunk", "frame"):
        spec = bg.make_spec(f_cur=3, f_kv=6, h=8, w=32, block_t=3, block_hw=(4, 4),
                            block_radius_hw=(1, 2), streaming=True)
        rows, stride, _ = bg.plan_rows(spec, mode)
        qw0, qwl, kw0, kwl, kw0a, kwla, _ = bg._PAIR_COLS[stride]
        seen = []
        for r, (w0, w1, e0, e1) in enumerate([(0, 16, 0, 24), (16, 32, 8, 32)]):
            sr = bg.strip_rows(rows, stride, w0, w1, e0, e1 - e0)
            back = sr.to(torch.int64).clone()
            back[:, qw0] += w0
            back[:, kw0] += e0
            back[:, kw0a] += e0
            back[:, stride - 1] = 32
            seen.append(back)
        got = sorted(map(tuple, torch.cat(seen).tolist()))
        assert got == sorted(map(tuple, rows.to(torch.int64).tolist())), mode
    with pytest.raises(ValueError, match="outside"):
        bg.strip_rows(rows, stride, 0, 16, 0, 16)   # no room for the halo
