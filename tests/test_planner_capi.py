"""Host logic and the C ABI, without a GPU."""
import ctypes
import re

import numpy as np
import pytest
import torch

from tests.golden_cases import PLAN_NAMES, spec_fields


@pytest.mark.parametrize("name", PLAN_NAMES)
def test_product_plan_rows_match_reference(srdit, golden, name):
    """The package's own planner reproduces the reference's params rows."""
    g = golden("plans")
    vals, mode = spec_fields(g, name)
    spec = srdit.blockgrid.WindowSpec(**{k: vals[k] for k in (
        "f_cur", "f_kv", "h", "w", "block_t", "bh", "bw", "rh", "rw", "hist", "rt",
        "chunk_frames", "streaming", "anchor_hw")})
    rows, stride, hr_base = srdit.blockgrid.plan_rows(spec, mode)
    np.testing.assert_array_equal(rows.numpy(), g[f"{name}.params"])
    meta = g[f"{name}.meta"]
    assert stride == meta[5] and hr_base == meta[4]


def test_make_spec_matches_recorded_specs(srdit, golden):
    """make_spec derives rt / hist the way mask_free_window_attention does."""
    g = golden("plans")
    cases = {
        "2k_4x4_r3_f12": dict(f_cur=3, f_kv=12, h=36, w=64, block_t=3, block_hw=(4, 4),
                              block_radius_hw=(3, 3), streaming=True),
        "hist_rt1": dict(f_cur=3, f_kv=9, h=12, w=16, block_t=3, block_hw=(4, 4),
                         block_radius_hw=(1, 2), block_radius_t=1, streaming=True),
        "parallel_causal": dict(f_cur=6, f_kv=6, h=8, w=8, block_t=3, block_hw=(4, 4),
                                block_radius_hw=(1, 1), causal_chunk_frames=3,
                                causal_kv_span=6),
    }
    for name, kw in cases.items():
        vals, _ = spec_fields(g, name)
        spec = srdit.blockgrid.make_spec(**kw)
        for k in ("f_cur", "f_kv", "rt", "hist", "chunk_frames", "streaming"):
            assert getattr(spec, k) == vals[k], (name, k)


def test_library_exports_every_header_symbol(srdit):
    L = srdit._lib.lib()
    syms = srdit._lib.header_symbols()
    assert len(syms) >= 8
    for s in syms:
        assert hasattr(L, s), s
    assert L.srdit_version() == 1


def test_header_structs_match_ctypes(srdit):
    """The ctypes mirrors have the C structs' field lists."""
    text = srdit._lib.HEADER.read_text()
    for cname, pyt in (("srdit_winattn_geom", srdit._lib.WinattnGeom),
                       ("srdit_winattn_tiling", srdit._lib.WinattnTiling)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), text, re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        names = re.findall(r"(\w+)\s*[,;]", body)
        assert names == [f[0] for f in pyt._fields_], cname


def test_capi_rejects_bad_arguments_without_touching_the_gpu(srdit):
    L = srdit._lib.lib()
    # null operands / negative sizes are rejected by host-side checks
    rc = L.srdit_fp8_gemm(None, None, None, None, None, None, 16, 16, 16, 16, 16, 16, 0,
                          None, 0, None, None, None, None)
    assert rc == -1
    rc = L.srdit_quant_rowwise(None, 256, 4, 256, None, None, 256, None, None)
    assert rc == -1
    rc = L.srdit_ln_mod_quant(None, 256, 4, 256, 1e-6, None, None, None, None, None, 256,
                              None, None)
    assert rc == -1
    t = srdit._lib.WinattnTiling()
    assert L.srdit_winattn_plan(None, 0, 19, 0, ctypes.byref(t)) == -1
    assert "invalid" in L.srdit_strerror(-1).decode()


@pytest.mark.parametrize("name,expect", [
    ("cfg1_8x8_r0", dict(bw_q=8, bh_q=8, qboxes_per_tile=2, m_tiles=2, bw_k=8, bh_k=8,
                         kboxes_per_tile=2)),
    ("2k_4x4_r3_f12", dict(bw_q=4, bh_q=4, qboxes_per_tile=8, m_tiles=1, bw_k=28, bh_k=4,
                           kboxes_per_tile=1)),
    ("2k_4x4_r3_f12_frame", dict(bw_a=28, bh_a=4, aboxes_per_tile=1, has_anchor=1)),
])
def test_kernel_tiling(srdit, golden, name, expect):
    g = golden("plans")
    params = torch.from_numpy(g[f"{name}.params"])
    meta = g[f"{name}.meta"]
    mode = spec_fields(g, name)[1]
    t = srdit.ops.winattn_plan(params, int(meta[5]), srdit.blockgrid.ANCHOR_MODES[mode])
    for k, v in expect.items():
        assert getattr(t, k) == v, (k, getattr(t, k), v)
    # every box is whole 1024-byte swizzle atoms and a tile is at most 128 rows
    for bw, bh, n in ((t.bw_q, t.bh_q, t.qboxes_per_tile), (t.bw_k, t.bh_k, t.kboxes_per_tile)):
        assert (bw * bh) % 8 == 0 and bw * bh * n <= 128


def test_install_swaps_the_reference_seam(srdit):
    class FakeAttentionModule:
        _run_blockgrid_triton = None
    srdit.attention.install(FakeAttentionModule)
    assert FakeAttentionModule._run_blockgrid_triton is srdit.attention.run_blockgrid_b200


def test_no_fallback_on_cpu_tensors(srdit):
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(srdit._lib.SrditError):
        srdit.ops.quant_rowwise(x)
    with pytest.raises(ValueError):
        srdit.attention.mask_free_window_attention(
            torch.zeros(1, 8, 1, 128), torch.zeros(1, 8, 1, 128), torch.zeros(1, 8, 1, 128),
            torch.tensor([[1, 2, 4]]), attn_impl="sdpa", block_t=1)


def test_visible_flops_config3(srdit):
    """Algorithmic FLOPs of the config-3 window attention (8x8, r0, f_kv=6)."""
    spec = srdit.blockgrid.make_spec(f_cur=3, f_kv=6, h=36, w=64, block_t=3, block_hw=(8, 8),
                                     block_radius_hw=(0, 0), streaming=True)
    rows, stride, _ = srdit.blockgrid.plan_rows(spec)
    fl = srdit.blockgrid.visible_flops(rows, stride, 24, 128)
    # 6912 queries, each sees 6 frames x its 8x8 (or 4x8 edge) block
    assert fl == 4 * 128 * 24 * sum(
        3 * qh * 8 * 6 * qh * 8 for qh in (8, 8, 8, 8, 4) for _ in range(8))


def test_rows_outside_the_grid_are_rejected(srdit, golden):
    g = golden("plans")
    params = torch.from_numpy(g["2k_4x4_r3_f6.params"]).clone()
    srdit.attention.check_rows(params, 19, f_cur=3, h=36, w=64, kv_frames=6)
    with pytest.raises(ValueError):
        srdit.attention.check_rows(params, 19, f_cur=3, h=32, w=64, kv_frames=6)
    with pytest.raises(ValueError):
        srdit.attention.check_rows(params, 19, f_cur=3, h=36, w=64, kv_frames=5)
    params[7, 11] += 1   # widen one KV cuboid past the grid edge
    params[7, 10] = 64 - params[7, 11] + 1
    with pytest.raises(ValueError):
        srdit.attention.check_rows(params, 19, f_cur=3, h=36, w=64, kv_frames=6)


@pytest.mark.parametrize("name", ["2k_4x4_r3_f6", "2k_4x4_r3_f12_frame", "2k_4x4_r3_f6_chunk",
                                  "odd_frame", "2k_8x8_r0_f6", "cfg1_4x4_r3"])
def test_window_pairs_round_trip_and_cover_the_same_pairs(srdit, golden, name):
    """Merging adjacent windows (pair_rows) keeps every window's visible set:
    unpair_rows restores the reference's rows exactly, the merged rows stay
    inside the grids, and the kernel's tile-pair count drops where it pays."""
    import importlib
    from tests.golden_cases import spec_fields
    bg = importlib.import_module("dreamx-creator_b200.blockgrid")
    attn = importlib.import_module("dreamx-creator_b200.attention")
    g = golden("plans")
    vals, mode = spec_fields(g, name)
    rows = torch.from_numpy(g[f"{name}.params"]).to(torch.int32)
    stride = int(g[f"{name}.meta"][5])
    merged, split = bg.pair_rows(rows, stride)
    assert torch.equal(bg.unpair_rows(merged, split, stride), rows)
    a_hw = vals["anchor_hw"] or (vals["h"], vals["w"]) if mode else None
    attn.check_rows(merged, stride, f_cur=vals["f_cur"], h=vals["h"], w=vals["w"],
                    kv_frames=vals["f_kv"], a_hw=a_hw, a_frames=vals["f_cur"] if mode else 0)
    if name.startswith("2k_4x4") or name == "cfg1_4x4_r3":
        assert merged.shape[0] * 2 == rows.shape[0]
        code = {None: 0, "chunk": 1, "frame": 2}[mode]
        t0 = srdit.ops.winattn_plan(rows, stride, code)
        t1 = srdit.ops.winattn_plan(merged, stride, code)
        assert bg.tile_pairs(merged, stride, t1) < 0.7 * bg.tile_pairs(rows, stride, t0)


@pytest.mark.parametrize("name,split", [("2k_4x4_r3_f6", 1), ("2k_4x4_r3_f12_frame", 1),
                                        ("2k_8x8_r0_f6", 0), ("cfg1_8x8_r0", 0)])
def test_split_kv_schedule_choice(srdit, golden, name, split):
    """The planner picks the split-KV schedule for items that average 12 KV
    tiles or more (the shipped 4x4 radius-3 windows, about 30), not for
    BASELINE's 8x8 windows (3 to 6 tiles per item)."""
    g = golden("plans")
    params = torch.from_numpy(g[f"{name}.params"])
    mode = spec_fields(g, name)[1]
    t = srdit.ops.winattn_plan(params, int(g[f"{name}.meta"][5]),
                               srdit.blockgrid.ANCHOR_MODES[mode])
    assert t.split_kv == split
