"""Oracle: block-grid window visibility and the int32 params rows.

Restates (test infrastructure only):
  * ``_blockgrid_neighbours`` / ``_blockgrid_axis_blocks``
    -- video_refiner/wan/modules/sr_dit/attention.py:244-290 (the spatial rule)
  * ``_BlockGridSpec.temporal_runs`` -- attention.py:442-512 (the temporal rule,
    chunk-anchored ``hist`` and legacy derived-``rt``)
  * ``_BlockGridSpec.anchor_*`` / ``_anchor_grid_stride`` -- attention.py:293-328, 417-440
  * ``build_plan`` -- video_refiner/wan/modules/sr_dit/blockgrid_triton.py:83-150
  * the op's spec construction -- attention.py:1499-1616
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

P_FRAME, P_PLAIN = 17, 19


def axis_blocks(size: int, block: int, radius: int):
    """Per-block (q0, qL, k0, kL) along one axis (attention.py:261-290)."""
    nb = (size + block - 1) // block
    out = []
    for b in range(nb):
        q0, q1 = b * block, min((b + 1) * block, size)
        lo, hi = max(0, b - radius), min(nb - 1, b + radius)
        k0, k1 = lo * block, min((hi + 1) * block, size)
        out.append((q0, q1 - q0, k0, k1 - k0))
    return out


def anchor_stride(h, w, bh, bw, anchor_hw):
    """attention.py:293-328."""
    if anchor_hw is None:
        return 1, 1
    ha, wa = int(anchor_hw[0]), int(anchor_hw[1])
    if ha <= 0 or wa <= 0 or h % ha or w % wa:
        raise ValueError("anchor grid must divide the query grid")
    sh, sw = h // ha, w // wa
    if bh % sh or bw % sw:
        raise ValueError("anchor stride must divide the block size")
    return sh, sw


@dataclass(frozen=True)
class Spec:
    """Fields of ``_BlockGridSpec`` (attention.py:348-415)."""
    f_cur: int
    f_kv: int
    h: int
    w: int
    block_t: int
    bh: int
    bw: int
    rh: int
    rw: int
    hist: int | None = None
    rt: int = 0
    chunk_frames: int | None = None
    streaming: bool = False
    query_grain: str = "grid"
    anchor_hw: tuple | None = None

    def h_blocks(self):
        return axis_blocks(self.h, self.bh, self.rh)

    def w_blocks(self):
        return axis_blocks(self.w, self.bw, self.rw)

    def anchor_h_blocks(self):
        s = anchor_stride(self.h, self.w, self.bh, self.bw, self.anchor_hw)[0]
        return [(a, b, c // s, d // s) for (a, b, c, d) in self.h_blocks()]

    def anchor_w_blocks(self):
        s = anchor_stride(self.h, self.w, self.bh, self.bw, self.anchor_hw)[1]
        return [(a, b, c // s, d // s) for (a, b, c, d) in self.w_blocks()]

    @property
    def anchor_grid(self):
        if self.anchor_hw is None:
            return self.h, self.w
        return int(self.anchor_hw[0]), int(self.anchor_hw[1])

    @property
    def one_query_run(self):
        return bool(self.streaming) or self.query_grain != "grid" or self.f_kv != self.f_cur

    def temporal_runs(self):
        """attention.py:442-512."""
        f_cur, f_kv = self.f_cur, self.f_kv
        if self.hist is not None:
            cf = int(self.chunk_frames) if self.chunk_frames else max(1, f_cur)
            if self.one_query_run or f_cur <= cf:
                runs = [(0, f_cur, max(0, f_kv - f_cur - self.hist), f_kv)]
            else:
                runs = [(c0, min(c0 + cf, f_cur), max(0, c0 - self.hist), min(f_kv, min(c0 + cf, f_cur)))
                        for c0 in range(0, f_cur, cf)]
        else:
            bt, rt = self.block_t, self.rt
            if self.one_query_run:
                runs = [(0, f_cur, max(0, f_kv - (rt + 1) * bt), f_kv)]
            elif f_cur < bt:
                runs = [(0, f_cur, 0, f_kv)]
            else:
                runs = [(i * bt, (i + 1) * bt, max(0, i - rt) * bt, (i + 1) * bt)
                        for i in range(f_cur // bt)]
        covered = sum(q1 - q0 for (q0, q1, _, _) in runs)
        if covered != f_cur or runs[0][0] != 0 or runs[-1][1] != f_cur:
            raise ValueError("temporal runs do not partition the query frames")
        return runs


def make_spec(f_cur, f_kv, h, w, *, block_t, block_hw, block_radius_hw, block_radius_t=None,
              streaming=False, causal_chunk_frames=None, causal_kv_span=None, anchor_hw=None):
    """The spec ``mask_free_window_attention`` builds (attention.py:1559-1616)."""
    bt = int(block_t)
    hist = None if block_radius_t is None else (2 * int(block_radius_t) + 1) * bt
    rt = (int(causal_kv_span) // bt - 1) if causal_kv_span is not None else (f_kv // bt - 1)
    rt = max(rt, 0)
    return Spec(f_cur=f_cur, f_kv=f_kv, h=h, w=w, block_t=bt, bh=int(block_hw[0]),
                bw=int(block_hw[1]), rh=int(block_radius_hw[0]), rw=int(block_radius_hw[1]),
                hist=hist, rt=rt,
                chunk_frames=None if causal_chunk_frames is None else int(causal_chunk_frames),
                streaming=streaming, anchor_hw=anchor_hw)


def build_plan(spec: Spec, anchor_mode=None):
    """The params rows of blockgrid_triton.py:83-150 (int32 [n_w, P])."""
    hb, wb = spec.h_blocks(), spec.w_blocks()
    hb_a, wb_a = spec.anchor_h_blocks(), spec.anchor_w_blocks()
    a_h, a_w = spec.anchor_grid
    runs = spec.temporal_runs()
    f_cur = spec.f_cur
    rows, lqs = [], []
    if anchor_mode == "frame":
        if len(runs) != 1 or runs[0][0] != 0 or runs[0][1] != f_cur:
            raise ValueError("frame anchor needs a single query run")
        _, _, kv0, kv1 = runs[0]
        for hi, (qh0, qhL, kh0, khL) in enumerate(hb):
            for wi, (qw0, qwL, kw0, kwL) in enumerate(wb):
                rows.append([qh0, qw0, qhL, qwL, kv0, kv1 - kv0, kh0, khL, kw0, kwL, f_cur,
                             hb_a[hi][2], hb_a[hi][3], wb_a[wi][2], wb_a[wi][3], a_h, a_w])
                lqs.append(f_cur * qhL * qwL)
    else:
        a_frames = f_cur if anchor_mode == "chunk" else 0
        for (q0, q1, kv0, kv1) in runs:
            for hi, (qh0, qhL, kh0, khL) in enumerate(hb):
                for wi, (qw0, qwL, kw0, kwL) in enumerate(wb):
                    rows.append([q0, q1 - q0, qh0, qw0, qhL, qwL, kv0, kv1 - kv0, kh0, khL,
                                 kw0, kwL, a_frames, hb_a[hi][2], hb_a[hi][3], wb_a[wi][2],
                                 wb_a[wi][3], a_h, a_w])
                    lqs.append((q1 - q0) * qhL * qwL)
    p2 = 1
    while p2 < max(lqs):
        p2 *= 2
    block_m = max(16, min(p2, 64))
    m_tiles = max((x + block_m - 1) // block_m for x in lqs)
    return {"params": np.asarray(rows, dtype=np.int32), "n_w": len(rows), "block_m": block_m,
            "m_tiles": m_tiles, "block_n": 64,
            "hr_base": (f_cur * a_h * a_w) if anchor_mode is not None else 0,
            "p_stride": P_FRAME if anchor_mode == "frame" else P_PLAIN}
