"""Oracle: execute a block-grid window plan on the CPU (test infrastructure only).

Follows the visibility the reference's fused kernels address
(video_refiner/wan/modules/sr_dit/blockgrid_triton.py:184-278 for the plain /
"chunk" rows, :281-389 for the per-frame-anchor rows): each window's query
cuboid attends an optional anchor prefix (every anchor frame of the chunk, or
only its own frame) followed by its HR KV cuboid, softmax over the union with
scale d^-0.5. Computed as an exact softmax in float64 (or float32) with torch on
the CPU, gathering the index sets explicitly -- the same sets the reference's
gather backend builds (attention.py:660-802).
"""
from __future__ import annotations

import numpy as np
import torch


def _cuboid(t0, tL, h0, hL, w0, wL, H, W, base=0):
    t = np.arange(t0, t0 + tL)[:, None, None]
    h = np.arange(h0, h0 + hL)[None, :, None]
    w = np.arange(w0, w0 + wL)[None, None, :]
    return (base + t * (H * W) + h * W + w).reshape(-1)


def window_index_sets(plan, f_cur, h, w, kv_w=None):
    """Yield (q_idx, kv_idx_list) per window: kv_idx_list is one index array per
    query sub-group (all query rows for plain rows; one per frame for frame rows),
    with its query index array. Indices address cat([anchor, HR]); the HR frames
    are h x kv_w tokens (default kv_w = w)."""
    kv_w = w if kv_w is None else kv_w
    params = np.asarray(plan["params"])
    hr_base = int(plan["hr_base"])
    frame = int(plan["p_stride"]) == 17
    for row in params.tolist():
        if frame:
            (qh0, qw0, qhL, qwL, kv0, kvL, kh0, khL, kw0, kwL, fc,
             kh0a, khLa, kw0a, kwLa, Ha, Wa) = row
            hr = _cuboid(kv0, kvL, kh0, khL, kw0, kwL, h, kv_w, base=hr_base)
            groups = []
            for t in range(fc):
                q = _cuboid(t, 1, qh0, qhL, qw0, qwL, h, w)
                a = _cuboid(t, 1, kh0a, khLa, kw0a, kwLa, Ha, Wa)
                groups.append((q, np.concatenate([a, hr])))
            yield groups
        else:
            (q0, qL, qh0, qw0, qhL, qwL, kv0, kvL, kh0, khL, kw0, kwL, af,
             kh0a, khLa, kw0a, kwLa, Ha, Wa) = row
            q = _cuboid(q0, qL, qh0, qhL, qw0, qwL, h, w)
            hr = _cuboid(kv0, kvL, kh0, khL, kw0, kwL, h, kv_w, base=hr_base)
            if af > 0:
                a = _cuboid(0, af, kh0a, khLa, kw0a, kwLa, Ha, Wa)
                kv = np.concatenate([a, hr])
            else:
                kv = hr
            yield [(q, kv)]


def run_plan(q, k_ext, v_ext, plan, *, f_cur, h, w, dtype=torch.float64, kv_w=None):
    """out[token] = softmax(q k^T * d^-0.5) v over each window's visible set.

    q: [f_cur*h*w, n, d]; k_ext/v_ext: [anchor + HR tokens, n, d] (torch CPU).
    Returns [f_cur*h*w, n, d] in ``dtype``.
    """
    q = q.to(dtype)
    k = k_ext.to(dtype)
    v = v_ext.to(dtype)
    n, d = q.shape[1], q.shape[2]
    out = torch.zeros(q.shape, dtype=dtype)
    scale = d ** -0.5
    for groups in window_index_sets(plan, f_cur, h, w, kv_w):
        for qi, kvi in groups:
            qi_t = torch.from_numpy(qi)
            kvi_t = torch.from_numpy(kvi)
            qg = q[qi_t].transpose(0, 1)            # [n, Lq, d]
            kg = k[kvi_t].transpose(0, 1)           # [n, Lkv, d]
            vg = v[kvi_t].transpose(0, 1)
            s = torch.matmul(qg, kg.transpose(1, 2)) * scale
            p = torch.softmax(s, dim=-1)
            out[qi_t] = torch.matmul(p, vg).transpose(0, 1)
    return out


def coverage(plan, f_cur, h, w):
    """Number of windows covering each query token (must be exactly 1 each)."""
    cnt = np.zeros(f_cur * h * w, dtype=np.int64)
    for groups in window_index_sets(plan, f_cur, h, w):
        for qi, _ in groups:
            np.add.at(cnt, qi, 1)
    return cnt


def visible_pairs(plan, f_cur, h, w, n_heads=1):
    """Sum over windows of Lq * Lkv (visible query-key pairs), times heads."""
    tot = 0
    for groups in window_index_sets(plan, f_cur, h, w):
        for qi, kvi in groups:
            tot += len(qi) * len(kvi)
    return tot * n_heads
