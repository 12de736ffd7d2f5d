"""Drop-in block-grid window attention on the B200 kernel.

Two seams of the reference (video_refiner/wan/modules/sr_dit/attention.py):

* ``run_blockgrid_b200`` has the signature of the reference's launcher
  ``run_blockgrid_triton(q, k_ext, v_ext, out, *, plan, f_cur, h, w, n, d,
  anchor_mode=None)`` (blockgrid_triton.py:392-422) and accepts the reference's
  own plan dicts. ``install(attention_module)`` points the reference's
  call-time-looked-up global ``_run_blockgrid_triton`` (attention.py:45-46) at it,
  so an unmodified reference model running ``attn_impl="triton"`` launches the
  B200 kernel.
* ``mask_free_window_attention`` has the reference op's signature
  (attention.py:1376-1395) and semantics -- validation, KV-cache concat and
  tail truncation, per-sample loop -- with ``attn_impl="b200"``.

Unsupported cases raise; nothing falls back to another backend.
"""
from __future__ import annotations

import torch

from . import _lib, blockgrid, ops

BLOCKGRID_IMPLS = ("b200",)


def check_rows(params: torch.Tensor, p_stride: int, *, f_cur, h, w, kv_frames, a_hw=None,
               a_frames=0, kv_w=None) -> None:
    """Every cuboid a params row addresses lies inside its tensor.

    The kernel addresses tokens straight from the rows, so this is the check that
    keeps a malformed plan from turning into an out-of-bounds store. ``kv_w``:
    the K/V frames' width when it differs from the query grid's ``w``.
    """
    kv_w = w if kv_w is None else kv_w
    p = params.to(torch.int64)
    if p.dim() != 2 or p.shape[1] != p_stride:
        raise ValueError(f"params rows must be [n_w, {p_stride}], got {tuple(p.shape)}")
    if p_stride == blockgrid.P_FRAME:
        q_t0, q_tL = torch.zeros_like(p[:, 0]), p[:, 10]
        q_h0, q_w0, qhL, qwL, kv0, kvL, kh0, khL, kw0, kwL = (p[:, i] for i in range(10))
        a_f = p[:, 10]
        kh0a, khLa, kw0a, kwLa = p[:, 11], p[:, 12], p[:, 13], p[:, 14]
    else:
        (q_t0, q_tL, q_h0, q_w0, qhL, qwL, kv0, kvL, kh0, khL, kw0, kwL, a_f,
         kh0a, khLa, kw0a, kwLa) = (p[:, i] for i in range(17))
    ok = ((q_t0 >= 0) & (q_tL > 0) & (q_t0 + q_tL <= f_cur) & (q_h0 >= 0) & (qhL > 0)
          & (q_h0 + qhL <= h) & (q_w0 >= 0) & (qwL > 0) & (q_w0 + qwL <= w)
          & (kv0 >= 0) & (kvL > 0) & (kv0 + kvL <= kv_frames) & (kh0 >= 0) & (khL > 0)
          & (kh0 + khL <= h) & (kw0 >= 0) & (kwL > 0) & (kw0 + kwL <= kv_w))
    if not bool(ok.all()):
        raise ValueError("a window params row addresses tokens outside the q/KV grids")
    if a_hw is not None:
        has = a_f > 0
        ok_a = (~has) | ((a_f <= a_frames) & (kh0a >= 0) & (khLa > 0) & (kh0a + khLa <= a_hw[0])
                         & (kw0a >= 0) & (kwLa > 0) & (kw0a + kwLa <= a_hw[1]))
        if not bool(ok_a.all()):
            raise ValueError("a window params row addresses anchor tokens outside the anchor")


# Merge horizontally adjacent windows into one launch row when that cuts the
# kernel's (query tile, KV tile) pairs below this fraction of the unmerged count
PAIR_GAIN = 0.85


def _plan_device_state(plan: dict, device: torch.device, anchor_mode, check_key, check_kw):
    """Device params + kernel tiling (+ the window-pair records), cached inside the
    plan dict per device; the rows are bounds-checked once per (device, tensor
    geometry). Returns (params_dev, tiling, n_rows, anchor mode, split_dev or None).

    Windows narrower than a query tile (the shipped 3x4x4 windows hold 48
    queries, 37% of a 128-row tile) run two at a time: the rows of two
    horizontally adjacent windows merge into one row over the union of their
    KV columns, and the kernel masks each query row to its own window's columns
    (``blockgrid.pair_rows``). The merge is used when it cuts the kernel's tile
    pairs enough; every query row still sees exactly its own window's keys."""
    key = ("b200", device)
    st = plan.get(key)
    if st is None:
        params = plan["params"]
        if not torch.is_tensor(params):
            params = torch.as_tensor(params)
        params = params.to(torch.int32).contiguous().cpu()
        stride = int(plan["p_stride"])
        mode = blockgrid.ANCHOR_MODES[anchor_mode]
        tiling = ops.winattn_plan(params, stride, mode)
        split_dev = None
        rows_p, split = blockgrid.pair_rows(params, stride)
        if rows_p.shape[0] < params.shape[0]:
            tiling_p = ops.winattn_plan(rows_p, stride, mode)
            if (blockgrid.tile_pairs(rows_p, stride, tiling_p)
                    < PAIR_GAIN * blockgrid.tile_pairs(params, stride, tiling)):
                params, tiling = rows_p, tiling_p
                split_dev = split.to(device)
        st = plan[key] = (params.to(device), tiling, params.shape[0], mode, split_dev, params,
                          set())
    if check_key not in st[6]:
        check_rows(st[5], int(plan["p_stride"]), **check_kw)
        st[6].add(check_key)
    return st[:5]


def _geom(q, k_hr, *, f_cur, h, w, n, d, kv_frames, kv_slot0=0, anchor=None, a_hw=None):
    g = _lib.WinattnGeom()
    g.q_frames, g.q_h, g.q_w = f_cur, h, w
    g.kv_h, g.kv_w = h, w
    g.kv_slots, g.kv_slot0 = kv_frames, kv_slot0
    if anchor is not None:
        g.a_h, g.a_w = a_hw
        g.a_frames = anchor.shape[0] // (a_hw[0] * a_hw[1])
        g.a_stride = anchor.stride(0)
    g.n_heads, g.head_dim = n, d
    g.q_stride = q.stride(0)
    g.kv_stride = k_hr.stride(0)
    g.o_stride = q.stride(0)
    g.scale = d ** -0.5
    return g


def run_blockgrid_b200(q, k_ext, v_ext, out, *, plan, f_cur, h, w, n, d, anchor_mode=None,
                       status=None):
    """Launch the B200 kernel for one sample; writes ``out`` and returns it.

    ``q``/``out``: [f_cur*h*w, n, d]; ``k_ext``/``v_ext``: ``cat([anchor, HR])``
    when an anchor is present (HR starts at ``plan["hr_base"]``), else the HR
    KV alone -- the layout the reference's launcher takes.
    """
    if d != 128:
        raise _lib.SrditError(f"the B200 window kernel supports head_dim 128, got {d}")
    for t in (q, k_ext, v_ext, out):
        if not t.is_contiguous():
            raise _lib.SrditError("q/k/v/out must be contiguous with a stride-1 head dim")
    hr_base = int(plan.get("hr_base", f_cur * h * w if anchor_mode is not None else 0))
    L = h * w
    if q.numel() != f_cur * L * n * d or out.shape != q.shape:
        raise ValueError("q/out must be [f_cur*h*w, n, d]")
    kf, vf = k_ext.view(-1, n * d), v_ext.view(-1, n * d)
    if kf.shape != vf.shape or kf.shape[0] < hr_base or (kf.shape[0] - hr_base) % L:
        raise ValueError("k_ext/v_ext must hold the anchor prefix plus whole HR frames")
    ka = va = None
    if anchor_mode is not None and hr_base > 0:
        ka, va = kf[:hr_base], vf[:hr_base]
    _launch(q.view(-1, n * d), kf[hr_base:], vf[hr_base:], out.view(-1, n * d), plan=plan,
            f_cur=f_cur, h=h, w=w, n=n, d=d, anchor_mode=anchor_mode, ka=ka, va=va,
            status=status)
    return out


def _launch(qf, k_hr, v_hr, of, *, plan, f_cur, h, w, n, d, anchor_mode, ka=None, va=None,
            k_hr2=None, v_hr2=None, status=None):
    """The kernel launch on [tokens, n*d] row views: the HR K/V (whole frames) and,
    for an anchored plan, the anchor K/V as separate tensors (the kernel reads
    each through its own tensor maps, so they need not be concatenated).
    ``k_hr2`` / ``v_hr2``: an optional second HR segment holding the frames that
    follow ``k_hr``'s (a cache and the current chunk in separate buffers)."""
    L = h * w
    kv_frames = k_hr.shape[0] // L
    seg1 = kv_frames
    if k_hr2 is not None:
        for t in (k_hr2, v_hr2):
            if (t is None or t.dtype != torch.bfloat16 or t.device != k_hr.device
                    or t.stride() != k_hr.stride() or t.shape[1] != k_hr.shape[1]):
                raise _lib.SrditError("the second K/V segment must match the first's "
                                      "dtype, device, width and token stride")
        if k_hr2.shape != v_hr2.shape or k_hr2.shape[0] % L:
            raise ValueError("the second K/V segment must hold whole frames")
        kv_frames += k_hr2.shape[0] // L
    a_hw = None
    a_frames = 0
    if ka is not None:
        p0 = plan["params"][0]
        a_hw = (int(p0[-2]), int(p0[-1]))
        a_frames = ka.shape[0] // (a_hw[0] * a_hw[1])
    params_dev, tiling, n_w, mode, split_dev = _plan_device_state(
        plan, qf.device, anchor_mode, (f_cur, h, w, kv_frames, a_hw, a_frames),
        dict(f_cur=f_cur, h=h, w=w, kv_frames=kv_frames, a_hw=a_hw, a_frames=a_frames))
    g = _geom(qf, k_hr, f_cur=f_cur, h=h, w=w, n=n, d=d, kv_frames=kv_frames, anchor=ka, a_hw=a_hw)
    g.o_stride = of.stride(0)
    g.col_split = None if split_dev is None else split_dev.data_ptr()
    if k_hr2 is not None:
        g.k_hr2, g.v_hr2, g.kv_split = k_hr2.data_ptr(), v_hr2.data_ptr(), seg1
    ops.winattn(qf, k_hr, v_hr, of, params_dev=params_dev, n_w=n_w,
                p_stride=int(plan["p_stride"]), anchor_mode=mode, geom=g, tiling=tiling,
                k_anchor=ka, v_anchor=va, status=status)


_PLAN_CACHE: dict = {}


def cached_plan(spec: blockgrid.WindowSpec, anchor_mode=None) -> dict:
    """Plan dict for ``spec`` (host rows + per-device kernel state), memoised."""
    key = (spec, anchor_mode)
    plan = _PLAN_CACHE.get(key)
    if plan is None:
        rows, stride, hr_base = blockgrid.plan_rows(spec, anchor_mode)
        plan = _PLAN_CACHE[key] = {"params": rows, "n_w": rows.shape[0], "p_stride": stride,
                                   "hr_base": hr_base}
    return plan


def frames_plan(spec1: blockgrid.WindowSpec, frames: int) -> dict:
    """Plan of ``frames`` independent 1-frame samples laid side by side in one
    chunk: the rows of the 1-frame spec ``spec1`` (no cache, no anchor) repeated
    once per frame, with the query and KV frame of every row offset by the frame
    index, so frame j attends to frame j only. This is the anchor harvest's
    batch of B = frames independent samples (causal_inference.py:456-460) run
    as one forward; memoised."""
    key = ("frames", spec1, int(frames))
    plan = _PLAN_CACHE.get(key)
    if plan is None:
        if spec1.f_cur != 1 or spec1.f_kv != 1:
            raise ValueError("frames_plan needs the spec of a 1-frame sample without a cache")
        rows, stride, _ = blockgrid.plan_rows(spec1, None)
        reps = []
        for j in range(int(frames)):
            r = rows.clone()
            r[:, 0] += j  # q_t0
            r[:, 6] += j  # kv_t0
            reps.append(r)
        rows = torch.cat(reps)
        plan = _PLAN_CACHE[key] = {"params": rows, "n_w": rows.shape[0], "p_stride": stride,
                                   "hr_base": 0}
    return plan


def install(attention_module) -> None:
    """Route the reference's ``attn_impl="triton"`` launches to the B200 kernel.

    ``attention_module`` is the reference's ``wan.modules.sr_dit.attention``;
    its ``_run_blockgrid_triton`` global is looked up at call time
    (attention.py:45-46), which is the seam swapped here.
    """
    attention_module._run_blockgrid_triton = run_blockgrid_b200


def _new_cache(ck, cv, k, v, kv_len, L):
    """The returned cache: the last ``kv_len`` frames of cat([cache, chunk]) (all of
    them when kv_len is None), as the reference returns it (attention.py:964-974).
    It is a view of the chunk when the chunk alone covers it; otherwise only the
    frames kept are copied."""
    total = k.shape[0] + (ck.shape[0] if ck is not None else 0)
    keep = total if kv_len is None else min(total, int(kv_len) * L)
    if ck is None or keep <= k.shape[0]:
        return k[k.shape[0] - keep:], v[v.shape[0] - keep:]
    tail = keep - k.shape[0]
    return (torch.cat([ck[ck.shape[0] - tail:], k], dim=0),
            torch.cat([cv[cv.shape[0] - tail:], v], dim=0))


def mask_free_window_attention(q, k, v, grid_sizes, pre_cache_k=None, pre_cache_v=None,
                               kv_len=None, anchor_k=None, anchor_v=None, anchor_align="frame",
                               anchor_window_scope="window", anchor_hw=None, anchor_keep=None,
                               attn_impl="b200", win_chunk=None, causal_chunk_frames=None,
                               causal_kv_span=None, block_t=None, block_hw=(4, 4),
                               block_radius_hw=(2, 2), block_radius_t=None):
    """The reference op (attention.py:1376-1648) on the B200 kernel.

    Returns ``(out [b, s_cur, n, d], new_cache_k, new_cache_v)``.
    """
    if str(attn_impl) not in BLOCKGRID_IMPLS:
        raise ValueError(f"attn_impl must be one of {BLOCKGRID_IMPLS}, got {attn_impl!r}.")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                       for t in (q, k, v, anchor_k, anchor_v)):
        raise RuntimeError("the B200 window kernel is forward-only; an input requires grad.")
    b, s_cur, n, d = q.shape
    anchor_given = anchor_k is not None or anchor_v is not None
    if anchor_given and (anchor_k is None or anchor_v is None):
        raise ValueError("mask_free_window_attention: anchor_k and anchor_v must be provided together.")
    if anchor_given and anchor_align not in ("frame", "chunk"):
        raise ValueError(f"anchor_align must be 'frame' or 'chunk', got {anchor_align!r}.")
    if anchor_given and anchor_window_scope != "window":
        raise ValueError("the B200 window kernel supports anchor_window_scope='window' only "
                         "(one spatial extent per params row, as the fused reference kernel).")
    outs, cks, cvs = [], [], []
    for i in range(b):
        f_cur, h, w = (int(x) for x in grid_sizes[i].tolist())
        if f_cur * h * w != s_cur:
            raise ValueError(f"grid {(f_cur, h, w)} inconsistent with s_cur={s_cur}")
        L = h * w
        cached = pre_cache_k is not None and pre_cache_v is not None
        kv_tokens = k.shape[1] + (pre_cache_k.shape[1] if cached else 0)
        f_kv = kv_tokens // L
        if f_kv * L != kv_tokens or (cached and pre_cache_k.shape[1] % L):
            raise ValueError("KV cache is not aligned to whole frames")
        a_hw = None if anchor_hw is None or tuple(int(x) for x in anchor_hw) == (h, w) \
            else (int(anchor_hw[0]), int(anchor_hw[1]))
        use_anchor = anchor_given
        if anchor_given:
            s_h, s_w = blockgrid.anchor_stride(h, w, int(block_hw[0]), int(block_hw[1]), a_hw)
            La = (h // s_h) * (w // s_w)
            if anchor_k.shape[1] != f_cur * La:
                raise ValueError(f"frame-aligned LQ-anchor needs {f_cur * La} tokens per sample, "
                                 f"got {anchor_k.shape[1]}.")
            if (causal_chunk_frames is not None and causal_kv_span is not None
                    and pre_cache_k is None and pre_cache_v is None):
                raise NotImplementedError("LQ-anchor in the parallel chunk-causal window path is "
                                          "not supported.")
            if anchor_keep is not None:
                keep = anchor_keep.view(-1)[i] if torch.is_tensor(anchor_keep) else anchor_keep[i]
                use_anchor = bool(keep)
        bt = int(block_t if block_t is not None else causal_chunk_frames)
        streaming = pre_cache_k is not None or pre_cache_v is not None or anchor_given
        if block_radius_t is None and not streaming and f_cur % bt != 0 and f_cur >= bt:
            raise ValueError(f"block-grid window attention needs f_cur ({f_cur}) to be a "
                             f"multiple of block_t ({bt}).")
        spec = blockgrid.make_spec(f_cur=f_cur, f_kv=f_kv, h=h, w=w, block_t=bt, block_hw=block_hw,
                                   block_radius_hw=block_radius_hw,
                                   block_radius_t=block_radius_t, streaming=streaming,
                                   causal_chunk_frames=causal_chunk_frames,
                                   causal_kv_span=causal_kv_span,
                                   anchor_hw=a_hw if anchor_given else None)
        mode = None if not use_anchor else ("frame" if anchor_align == "frame" else "chunk")
        plan = cached_plan(spec, mode)
        if d != 128:
            raise _lib.SrditError(f"the B200 window kernel supports head_dim 128, got {d}")
        q_i = q[i].contiguous()
        out_i = torch.empty_like(q_i)
        # the anchor goes to the kernel as its own tensors: no cat([anchor, HR])
        # copy of the whole window K/V, which the reference's launcher layout needs
        ka = va = None
        if use_anchor:
            ka = anchor_k[i].contiguous().view(-1, n * d)
            va = anchor_v[i].contiguous().view(-1, n * d)
        # the cached frames and the current chunk go to the kernel as two K/V
        # segments: no cat([cache, chunk]) copy for the attention itself
        k_cur = k[i].contiguous().view(-1, n * d)
        v_cur = v[i].contiguous().view(-1, n * d)
        k2 = v2 = None
        if cached and pre_cache_k.shape[1] > 0:
            k_hr = pre_cache_k[i].contiguous().view(-1, n * d)
            v_hr = pre_cache_v[i].contiguous().view(-1, n * d)
            k2, v2 = k_cur, v_cur
        else:
            k_hr, v_hr = k_cur, v_cur
        _launch(q_i.view(-1, n * d), k_hr, v_hr, out_i.view(-1, n * d), plan=plan, f_cur=f_cur,
                h=h, w=w, n=n, d=d, anchor_mode=mode, ka=ka, va=va, k_hr2=k2, v_hr2=v2)
        outs.append(out_i)
        ck, cv = _new_cache(pre_cache_k[i] if cached else None,
                            pre_cache_v[i] if cached else None, k[i], v[i], kv_len, L)
        cks.append(ck)
        cvs.append(cv)
    out = torch.stack(outs, dim=0)
    if b == 1:
        return out, cks[0].unsqueeze(0), cvs[0].unsqueeze(0)
    return out, torch.stack(cks, dim=0), torch.stack(cvs, dim=0)
