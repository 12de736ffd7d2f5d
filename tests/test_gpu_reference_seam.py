"""The reference's own window-attention op through the launcher seam (GPU required).

The reference's ``mask_free_window_attention`` (attention.py:1376-1648) reaches
its Triton kernel through the module global ``_run_blockgrid_triton``
(attention.py:45-46), looked up at call time. ``attention.install`` points that
global at ``run_blockgrid_b200``. These tests run the reference op three ways
on the same seeded bf16 inputs:

- ``attn_impl="triton"`` with the stock launcher (the reference's Triton kernel,
  blockgrid_triton.py:184-422);
- ``attn_impl="triton"`` with the B200 launcher installed at the seam;
- ``attn_impl="sdpa"`` on the same inputs widened to fp32 (the reference's
  gather path, attention.py:660-802): the fp32 truth both are measured against.

Tolerances are the window-attention bar of the path's spec: bf16 max-abs
<= 2e-2 and relative (Frobenius) error <= 5e-3, against the reference kernel and
against the fp32 truth.

The reference is imported from its install under ``baseline/_ref`` (the
repository's reference arm); where that install is absent the tests skip.
"""
import pathlib
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = pathlib.Path(__file__).resolve().parents[1] / "baseline" / "_ref"
MAX_ABS, REL = 2e-2, 5e-3


@pytest.fixture(scope="module")
def ref_attention():
    if not (REF / "wan" / "modules" / "sr_dit" / "attention.py").exists():
        pytest.skip("the reference is not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from wan.modules.sr_dit import attention
    return attention


# (name, f_cur, f_cache, h, w, heads, block_hw, radius_hw, anchor_align)
CASES = [
    ("cfg1_8x8_r0", 3, 0, 18, 32, 24, (8, 8), (0, 0), None),
    ("cfg1_4x4_r3", 3, 0, 18, 32, 24, (4, 4), (3, 3), None),
    ("2k_8x8_r0_fkv6", 3, 3, 36, 64, 4, (8, 8), (0, 0), None),
    ("2k_4x4_r3_fkv6_frame", 3, 3, 36, 64, 2, (4, 4), (3, 3), "frame"),
    ("2k_4x4_r3_fkv6_chunk", 3, 3, 36, 64, 2, (4, 4), (3, 3), "chunk"),
]


def _err(a, b):
    d = (a.float() - b.float()).abs()
    return d.max().item(), (d.norm() / b.float().norm()).item()


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_reference_op_through_seam(srdit, cuda_device, ref_attention, case):
    name, f_cur, f_cache, h, w, n, bhw, rhw, align = case
    L, d = h * w, 128
    g = torch.Generator(device=cuda_device).manual_seed(sum(name.encode()))

    def rnd(tokens):
        return torch.randn(1, tokens, n, d, device=cuda_device, generator=g).to(torch.bfloat16)

    q, k, v = rnd(f_cur * L), rnd(f_cur * L), rnd(f_cur * L)
    ck, cv = (rnd(f_cache * L), rnd(f_cache * L)) if f_cache else (None, None)
    ak, av = (rnd(f_cur * L), rnd(f_cur * L)) if align else (None, None)
    grid = torch.tensor([[f_cur, h, w]])

    def run(impl, cast=lambda t: t):
        kw = dict(anchor_k=cast(ak), anchor_v=cast(av), anchor_align=align) if align else {}
        return ref_attention.mask_free_window_attention(
            cast(q), cast(k), cast(v), grid,
            pre_cache_k=None if ck is None else cast(ck),
            pre_cache_v=None if cv is None else cast(cv), kv_len=f_cache,
            attn_impl=impl, block_t=3, block_hw=bhw, block_radius_hw=rhw, **kw)[0]

    stock = ref_attention._run_blockgrid_triton
    with torch.no_grad():
        out_triton = run("triton")
        srdit.attention.install(ref_attention)
        try:
            assert ref_attention._run_blockgrid_triton is srdit.attention.run_blockgrid_b200
            out_b200 = run("triton")
        finally:
            ref_attention._run_blockgrid_triton = stock
        truth = run("sdpa", cast=lambda t: t.float())
    torch.cuda.synchronize()
    assert out_b200.dtype == torch.bfloat16 and out_b200.shape == out_triton.shape

    e_kernel = _err(out_b200, out_triton)
    e_b200 = _err(out_b200, truth)
    e_triton = _err(out_triton, truth)
    assert e_kernel[0] <= MAX_ABS and e_kernel[1] <= REL, (name, "vs reference kernel", e_kernel)
    assert e_b200[0] <= MAX_ABS and e_b200[1] <= REL, (name, "vs fp32 truth", e_b200)
    # the reference kernel meets the same bar, so the bar is not loose for it
    assert e_triton[0] <= MAX_ABS and e_triton[1] <= REL, (name, "reference vs truth", e_triton)
