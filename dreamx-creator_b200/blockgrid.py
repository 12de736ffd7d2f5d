"""Block-grid window geometry -> int32 params rows for the window kernel.

The visibility rule has to be the reference's exactly, so this module states the
same rules (video_refiner/wan/modules/sr_dit/attention.py):
  * spatial: query blocks tile each axis; block b sees blocks [b-r, b+r] clamped
    to the grid, one contiguous interval (attention.py:244-290);
  * temporal: the chunk-anchored ``hist`` rule or the legacy derived-``rt`` rule
    (``_BlockGridSpec.temporal_runs``, attention.py:442-512);
  * the anchor's own coarser grid (attention.py:293-328, 417-440);
and emits rows in the reference's params layouts (blockgrid_triton.py:77-80),
so a plan built here and a plan built by the reference's ``build_plan`` are
interchangeable at the launcher seam. What differs is the kernel tiling: the
B200 kernel packs whole (frame x rows x cols) boxes into 128-row tiles, which
``srdit_winattn_plan`` derives from the same rows.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

P_FRAME, P_PLAIN = 17, 19
ANCHOR_MODES = {None: 0, "chunk": 1, "frame": 2}


def axis_extents(size: int, block: int, radius: int):
    """[(q_start, q_len, kv_start, kv_len)] per block along one axis."""
    n_blocks = -(-size // block)
    spans = []
    for b in range(n_blocks):
        q_start = b * block
        q_len = min(q_start + block, size) - q_start
        first = max(b - radius, 0)
        last = min(b + radius, n_blocks - 1)
        kv_start = first * block
        kv_len = min((last + 1) * block, size) - kv_start
        spans.append((q_start, q_len, kv_start, kv_len))
    return spans


def anchor_stride(h, w, bh, bw, anchor_hw):
    if anchor_hw is None:
        return 1, 1
    h_a, w_a = int(anchor_hw[0]), int(anchor_hw[1])
    if h_a <= 0 or w_a <= 0:
        raise ValueError(f"LQ-anchor token grid {(h_a, w_a)}: both sides need at least one token")
    if h % h_a or w % w_a:
        raise ValueError(f"LQ-anchor token grid {(h_a, w_a)} is not a whole-number thinning of the "
                         f"{h}x{w} query grid")
    s_h, s_w = h // h_a, w // w_a
    if bh % s_h or bw % s_w:
        raise ValueError(f"{bh}x{bw} query blocks cannot be thinned by the anchor step "
                         f"{(s_h, s_w)}: a block would straddle anchor tokens")
    return s_h, s_w


@dataclass(frozen=True)
class WindowSpec:
    """One window geometry; the fields mean what ``_BlockGridSpec``'s do."""
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
    anchor_hw: tuple | None = None

    @property
    def single_query_run(self) -> bool:
        return self.streaming or self.f_kv != self.f_cur

    def frame_runs(self):
        """[(q_f0, q_f1, kv_f0, kv_f1)] partitioning the query frames."""
        f_cur, f_kv = self.f_cur, self.f_kv
        if self.hist is not None:
            cf = self.chunk_frames or max(1, f_cur)
            if self.single_query_run or f_cur <= cf:
                runs = [(0, f_cur, max(0, f_kv - f_cur - self.hist), f_kv)]
            else:
                runs = []
                for c0 in range(0, f_cur, cf):
                    c1 = min(c0 + cf, f_cur)
                    runs.append((c0, c1, max(0, c0 - self.hist), min(f_kv, c1)))
        else:
            bt, rt = self.block_t, self.rt
            if self.single_query_run:
                runs = [(0, f_cur, max(0, f_kv - (rt + 1) * bt), f_kv)]
            elif f_cur < bt:
                runs = [(0, f_cur, 0, f_kv)]
            else:
                runs = [(i * bt, (i + 1) * bt, max(0, i - rt) * bt, (i + 1) * bt)
                        for i in range(f_cur // bt)]
        if sum(b - a for a, b, _, _ in runs) != f_cur or runs[0][0] != 0 or runs[-1][1] != f_cur:
            raise ValueError(f"the {f_cur} query frames do not split into whole temporal blocks of "
                             f"{self.block_t} (runs {runs})")
        return runs

    def anchor_grid(self):
        if self.anchor_hw is None:
            return self.h, self.w
        return int(self.anchor_hw[0]), int(self.anchor_hw[1])


def make_spec(*, f_cur, f_kv, h, w, block_t, block_hw, block_radius_hw, block_radius_t=None,
              streaming=False, causal_chunk_frames=None, causal_kv_span=None,
              anchor_hw=None) -> WindowSpec:
    """The spec the op derives from its arguments (attention.py:1559-1616)."""
    bt = int(block_t)
    if bt <= 0:
        raise ValueError(f"block_t must be positive, got {bt}.")
    hist = None if block_radius_t is None else (2 * int(block_radius_t) + 1) * bt
    span = int(causal_kv_span) if causal_kv_span is not None else int(f_kv)
    return WindowSpec(f_cur=int(f_cur), f_kv=int(f_kv), h=int(h), w=int(w), block_t=bt,
                      bh=int(block_hw[0]), bw=int(block_hw[1]), rh=int(block_radius_hw[0]),
                      rw=int(block_radius_hw[1]), hist=hist, rt=max(span // bt - 1, 0),
                      chunk_frames=None if causal_chunk_frames is None else int(causal_chunk_frames),
                      streaming=bool(streaming), anchor_hw=anchor_hw)


def plan_rows(spec: WindowSpec, anchor_mode=None):
    """Params rows in the reference layout: (int32 [n_w, P], p_stride, hr_base)."""
    hb = axis_extents(spec.h, spec.bh, spec.rh)
    wb = axis_extents(spec.w, spec.bw, spec.rw)
    s_h, s_w = anchor_stride(spec.h, spec.w, spec.bh, spec.bw, spec.anchor_hw)
    h_a, w_a = spec.anchor_grid()
    runs = spec.frame_runs()
    rows = []
    if anchor_mode == "frame":
        if len(runs) != 1 or runs[0][:2] != (0, spec.f_cur):
            raise ValueError(f"a frame-aligned anchor pairs query frame t with anchor frame t, which "
                             f"needs all {spec.f_cur} query frames in one run (got {runs})")
        kv0, kv1 = runs[0][2:]
        for (qh0, qhL, kh0, khL) in hb:
            for (qw0, qwL, kw0, kwL) in wb:
                rows.append([qh0, qw0, qhL, qwL, kv0, kv1 - kv0, kh0, khL, kw0, kwL, spec.f_cur,
                             kh0 // s_h, khL // s_h, kw0 // s_w, kwL // s_w, h_a, w_a])
        stride = P_FRAME
    elif anchor_mode in (None, "chunk"):
        a_frames = spec.f_cur if anchor_mode == "chunk" else 0
        for (q0, q1, kv0, kv1) in runs:
            for (qh0, qhL, kh0, khL) in hb:
                for (qw0, qwL, kw0, kwL) in wb:
                    rows.append([q0, q1 - q0, qh0, qw0, qhL, qwL, kv0, kv1 - kv0, kh0, khL, kw0,
                                 kwL, a_frames, kh0 // s_h, khL // s_h, kw0 // s_w, kwL // s_w,
                                 h_a, w_a])
        stride = P_PLAIN
    else:
        raise ValueError(f"anchor_mode must be None, 'chunk' or 'frame', got {anchor_mode!r}.")
    hr_base = spec.f_cur * h_a * w_a if anchor_mode is not None else 0
    return torch.tensor(rows, dtype=torch.int32), stride, hr_base


def visible_flops(params: torch.Tensor, p_stride: int, n_heads: int, head_dim: int) -> int:
    """4*d*heads*sum(Lq*Lkv) over visible query-key pairs (no tile padding)."""
    p = params.tolist()
    tot = 0
    for r in p:
        if p_stride == P_FRAME:
            qhL, qwL, kvL, khL, kwL, fc, khLa, kwLa = r[2], r[3], r[5], r[7], r[9], r[10], r[12], r[14]
            tot += fc * qhL * qwL * (kvL * khL * kwL + khLa * kwLa)
        else:
            qL, qhL, qwL, kvL, khL, kwL, af, khLa, kwLa = r[1], r[4], r[5], r[7], r[9], r[11], r[12], r[14], r[16]
            tot += qL * qhL * qwL * (kvL * khL * kwL + af * khLa * kwLa)
    return 4 * head_dim * n_heads * tot


# Params-row columns of the fields a window pair merges, per row layout:
# (q_w0, qwL, kw0, kwL, kw0_a, kwL_a, anchor frames); the others must agree.
_PAIR_COLS = {P_PLAIN: (3, 5, 10, 11, 15, 16, 12), P_FRAME: (1, 3, 8, 9, 13, 14, 10)}
SPLIT_FIELDS = 9


def pair_rows(params: torch.Tensor, p_stride: int):
    """Merge horizontally adjacent windows into one row each: (rows, split).

    Rows i and i + 1 merge when window B = row i + 1 starts where window A =
    row i ends (B.q_w0 == A.q_w0 + A.qwL) and everything but their column
    extents agrees (query frames and rows, KV frames and rows, anchor frames
    and rows). The merged row is A's with the query columns of both and the
    union of their KV (and anchor) columns; ``split`` [n, SPLIT_FIELDS] int32
    records, per merged row, {q_split, hr_lo_a, hr_hi_a, hr_lo_b, hr_hi_b,
    an_lo_a, an_hi_a, an_lo_b, an_hi_b}: query columns [0, q_split) are A's,
    and each window keeps seeing only its own KV / anchor columns (relative to
    the merged row's kw0 / kw0_a). Rows that do not merge keep q_split 0.
    The merged rows are rows of the same layout and cover the same tokens, so
    they pass the same bounds checks; the kernel masks per query row.
    """
    qw0, qwl, kw0, kwl, kw0a, kwla, _ = _PAIR_COLS[p_stride]
    rows = params.to(torch.int64).tolist()
    keep = [i for i in range(p_stride) if i not in (qw0, qwl, kw0, kwl, kw0a, kwla)]
    out, split = [], []
    i = 0
    while i < len(rows):
        a = rows[i]
        b = rows[i + 1] if i + 1 < len(rows) else None
        ok = (b is not None and b[qw0] == a[qw0] + a[qwl] and b[kw0] >= a[kw0]
              and b[kw0] + b[kwl] >= a[kw0] + a[kwl] and all(a[k] == b[k] for k in keep))
        # the anchor columns merge the same way (the reference fills them in
        # rows without an anchor too, so the merge stays exactly invertible)
        if ok:
            ok = b[kw0a] >= a[kw0a] and b[kw0a] + b[kwla] >= a[kw0a] + a[kwla]
        if not ok:
            out.append(a)
            split.append([0] * SPLIT_FIELDS)
            i += 1
            continue
        u = list(a)
        u[qwl] = a[qwl] + b[qwl]
        u[kwl] = b[kw0] + b[kwl] - a[kw0]
        u[kwla] = b[kw0a] + b[kwla] - a[kw0a]
        rec = [a[qwl], 0, a[kwl], b[kw0] - a[kw0], b[kw0] - a[kw0] + b[kwl],
               0, a[kwla], b[kw0a] - a[kw0a], b[kw0a] - a[kw0a] + b[kwla]]
        out.append(u)
        split.append(rec)
        i += 2
    return (torch.tensor(out, dtype=torch.int32).reshape(-1, p_stride),
            torch.tensor(split, dtype=torch.int32).reshape(-1, SPLIT_FIELDS))


def tile_pairs(params: torch.Tensor, p_stride: int, tiling) -> int:
    """(query tile, KV tile) pairs the window kernel walks for these rows with
    this tiling: its work in units of the per-tile softmax + MMA step."""
    frame = p_stride == P_FRAME
    total = 0
    for r in params.to(torch.int64).tolist():
        if frame:
            q_tL, qhL, kv_tL, khL, a_f, khL_a = r[10], r[2], r[5], r[7], r[10], r[12]
        else:
            q_tL, qhL, kv_tL, khL, a_f, khL_a = r[1], r[4], r[7], r[9], r[12], r[14]
        hq = -(-qhL // tiling.bh_q)
        m_tiles = -(-(q_tL * hq) // tiling.qboxes_per_tile)
        kv = -(-(kv_tL * -(-khL // tiling.bh_k)) // tiling.kboxes_per_tile)
        if tiling.has_anchor and a_f > 0:
            per_frame = -(-(-(-khL_a // tiling.bh_a)) // tiling.aboxes_per_tile)
            # a frame-aligned anchor: each query tile sees the anchor frames of
            # its own query frames; a chunk anchor: every anchor frame
            kv += per_frame * (min(a_f, -(-tiling.qboxes_per_tile // hq)) if frame else a_f)
        total += m_tiles * kv
    return total


def strip_rows(params: torch.Tensor, p_stride: int, w_lo: int, w_hi: int, kv_lo: int,
               kv_w: int) -> torch.Tensor:
    """The rows of the windows whose query columns lie in [w_lo, w_hi) of the full
    grid, in the coordinates of a strip that holds those query columns and the
    K/V (and anchor) columns [kv_lo, kv_lo + kv_w): query column c becomes
    c - w_lo, KV and anchor columns c - kv_lo, and the anchor grid is kv_w wide.

    Every window must lie wholly inside or outside the strip, every kept row's
    KV columns inside [kv_lo, kv_lo + kv_w), and the anchor on the query's own
    token grid (anchor step 1, so its columns are the KV columns' numbering)."""
    qw0, qwl, kw0, kwl, kw0a, kwla, _ = _PAIR_COLS[p_stride]
    wa = p_stride - 1   # the anchor grid's width, last field of both layouts
    p = params.to(torch.int64)
    if p.numel() and not (torch.equal(p[:, kw0a], p[:, kw0]) and torch.equal(p[:, kwla], p[:, kwl])):
        raise ValueError("a strip's rows need the anchor on the query token grid (step 1)")
    inside = (p[:, qw0] >= w_lo) & (p[:, qw0] + p[:, qwl] <= w_hi)
    touches = (p[:, qw0] < w_hi) & (p[:, qw0] + p[:, qwl] > w_lo)
    if bool((touches & ~inside).any()):
        raise ValueError(f"a window crosses the edge of the strip [{w_lo}, {w_hi})")
    r = p[inside].clone()
    r[:, qw0] -= w_lo
    r[:, kw0] -= kv_lo
    r[:, kw0a] -= kv_lo
    r[:, wa] = kv_w
    if bool(((r[:, kw0] < 0) | (r[:, kw0] + r[:, kwl] > kv_w)).any()):
        raise ValueError(f"a window of the strip sees columns outside [{kv_lo}, {kv_lo + kv_w})")
    return r.to(torch.int32)


def unpair_rows(rows: torch.Tensor, split: torch.Tensor, p_stride: int) -> torch.Tensor:
    """The per-window rows that ``pair_rows`` merged (its inverse)."""
    qw0, qwl, kw0, kwl, kw0a, kwla, _ = _PAIR_COLS[p_stride]
    out = []
    for u, rec in zip(rows.to(torch.int64).tolist(), split.to(torch.int64).tolist()):
        if rec[0] == 0:
            out.append(u)
            continue
        a, b = list(u), list(u)
        a[qwl] = rec[0]
        b[qw0], b[qwl] = u[qw0] + rec[0], u[qwl] - rec[0]
        a[kw0], a[kwl] = u[kw0] + rec[1], rec[2] - rec[1]
        b[kw0], b[kwl] = u[kw0] + rec[3], rec[4] - rec[3]
        a[kw0a], a[kwla] = u[kw0a] + rec[5], rec[6] - rec[5]
        b[kw0a], b[kwla] = u[kw0a] + rec[7], rec[8] - rec[7]
        out += [a, b]
    return torch.tensor(out, dtype=torch.int32).reshape(-1, p_stride)
