"""Tensor-parallel SR-DiT forward: one process per GPU, heads and FFN sharded.

The reference's refiner runs on one GPU; its only tensor-parallel code is
DTensor-aware (``WanLayerNorm`` re-gathers a feature-sharded input,
video_refiner/wan/modules/sr_dit/models.py:455-496; the modulation becomes a
DTensor, :1243-1252). This module shards the block the Megatron way, with a
sequence-parallel residual stream between the sharded Linears:

  rank r of P holds heads [r*H/P, (r+1)*H/P) and FFN columns [r*F/P, (r+1)*F/P),
  and token rows [r*M/P, (r+1)*M/P) of the residual stream x.

Per block, per rank (Dl = D/P, Fl = F/P):

  ln_mod_quant(x_r)                  -> e4m3 [M/P, D]  -- all-gather -> [M, D]
  QKV (column-parallel, local heads) -> [M, 3*Dl]
  row sum-of-squares of q, k slices  -- all-reduce    -> full-width RMSNorm
  rms_rope, window attention (local heads, local K/V ring)
  row max|att| of the slice          -- all-reduce max -> per-token fp8 scale
  o (row-parallel, K = Dl)           -> bf16 partial [M, D] -- reduce-scatter
  residual(x_r, sum + bias, gate)
  (cross attention and FFN the same way; ffn.0's GELU amax is all-reduced)

Row-parallel weights are quantised per output channel over the FULL input
width before slicing, so every rank uses the reference's per-channel scales;
column-parallel weights are sliced by output rows, which keeps theirs exact.
The e4m3 inputs of the row-parallel Linears (attention outputs, the FFN
hidden) are scaled per token over the rank's own column slice
(``local_scales=True``, the default): each partial product is then exactly
the product of its own quantised slice, and the reduce-scatter sums them as
before, with no all-reduce of a per-token max in between (three of the five
per-block synchronisation points). The scale is finer-grained than one GPU's
full-row scale, never coarser. ``local_scales=False`` all-reduces the max so
each partial is the one-GPU product restricted to a K slice. What differs
from one GPU either way is the fp32 summation order, the bf16 rounding of each
rank's partial before the sum and, with local scales, the quantisation grid of
the row-parallel inputs.

Collectives go through ``TPComm`` (NCCL via torch.distributed). Every rank
issues the same collectives in the same order.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops
from .fp8_linear import quantize_weight
from .model import SRDiT, SRDiTConfig


class TPComm:
    """The collectives of the tensor-parallel forward, on one process group.

    fp8 buffers travel as bytes (the collectives only move them)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    @staticmethod
    def _bytes(t):
        return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t

    def all_gather(self, out, inp):
        dist.all_gather_into_tensor(self._bytes(out), self._bytes(inp), group=self.group)

    def reduce_scatter(self, out, inp):
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=self.group)

    def all_reduce_sum(self, t):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def all_reduce_max(self, t):
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)


class PeerComm(TPComm):
    """``TPComm`` plus symmetric peer buffers for the fused kernels.

    Each rank allocates one region and maps every peer's region (CUDA IPC):

      gather q [M, D] e4m3, gather s [M] fp32   all-gather target: each rank's LN
                                               kernel writes its own rows, the
                                               copy engines push them to the peers
      rs  [P, M/P, D] bf16                     reduce-scatter receive slots, one per
                                               source rank
      ar  2 x [P, n_ar] fp32                   all-reduce receive areas (alternating
                                               between calls)
      flags 3 x [8] uint32                     counters (gather / rs / ar), one per
                                               source rank

    Counters only grow; ``expected`` values are tracked here, identically on
    every rank, since all ranks issue the same kernels in the same order. The
    buffers are sized on first use for a chunk of M tokens (a collective step:
    every rank must reach it).

    Reuse is safe with single buffers for gather and rs: a rank writes a peer's
    gather rows (or rs slot) again only after it consumed that peer's next
    contribution, which the peer produces only after it finished reading the
    previous one. The all-reduce has no such step in between, hence two areas.
    """

    N_FLAG_SETS = 3   # gather, rs, ar

    def __init__(self, group=None, push="sm"):
        """``push``: how a rank's LN rows reach the peers' gather buffers -- "sm":
        the LN kernel stores them over NVLink itself and its last CTA signals;
        "ce": the copy engines push them on a side stream (one copy per peer)."""
        super().__init__(group)
        if push not in ("sm", "ce"):
            raise ValueError(f"push must be 'sm' or 'ce', not {push!r}")
        self.push = push
        self.key = None
        self.region = None
        self.peer_bases = []

    def setup(self, M, D, device):
        key = (M, D)
        if self.key == key:
            return
        if self.key is not None:
            raise _lib.SrditError("PeerComm buffers are sized for one chunk shape per model")
        P = self.world
        if M % P or (M // P) % 32:
            raise _lib.SrditError(f"fused tensor parallelism needs M/P a multiple of 32 "
                                  f"(M={M}, P={P})")
        Ml = M // P
        self.M, self.D, self.Ml = M, D, Ml
        self.n_ar = 2 * M + 4096
        al = lambda n: (n + 255) // 256 * 256  # noqa: E731
        sizes = [("gq", M * D), ("gs", 4 * M), ("rs", 2 * P * Ml * D),
                 ("ar0", 4 * P * self.n_ar), ("ar1", 4 * P * self.n_ar),
                 ("flags", 4 * 8 * self.N_FLAG_SETS)]
        self.off = {}
        total = 0
        for name, n in sizes:
            self.off[name] = total
            total += al(n)
        self.region = torch.zeros(total, dtype=torch.uint8, device=device)
        handle, offset = ops.ipc_handle(self.region)
        allh = [None] * P
        dist.all_gather_object(allh, (handle, offset), group=self.group)
        bases = []
        for d, (h, o) in enumerate(allh):
            if d == self.rank:
                bases.append(self.region.data_ptr())
            else:
                mapped = ops.ipc_open(h)
                self.peer_bases.append(mapped)
                bases.append(mapped + o)
        self.bases = bases
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)   # every region mapped and zeroed before first use
        r = self.region
        self.gq = r[self.off["gq"]:self.off["gq"] + M * D].view(torch.float8_e4m3fn).view(M, D)
        self.gs = r[self.off["gs"]:self.off["gs"] + 4 * M].view(torch.float32)
        self.rs = r[self.off["rs"]:self.off["rs"] + 2 * P * Ml * D].view(torch.bfloat16) \
            .view(P, Ml, D)
        addr = lambda name, extra=0: [b + self.off[name] + extra for b in bases]  # noqa: E731
        self.t_ar = [ops.peer_ptrs(addr("ar0")), ops.peer_ptrs(addr("ar1"))]
        self.t_flags = [ops.peer_ptrs(addr("flags", 32 * k)) for k in range(self.N_FLAG_SETS)]
        self.my_flags = [bases[self.rank] + self.off["flags"] + 32 * k
                         for k in range(self.N_FLAG_SETS)]
        self.rs_slot_addrs = [b + self.off["rs"] + self.rank * Ml * D * 2 for b in bases]
        # this rank's rows inside every rank's gather buffers (push targets)
        self.t_gq_rows = ops.peer_ptrs(addr("gq", self.rank * Ml * D))
        self.t_gs_rows = ops.peer_ptrs(addr("gs", self.rank * Ml * 4))
        self.side = torch.cuda.Stream(device)
        self.ev_ln = torch.cuda.Event()
        self.ev_push = torch.cuda.Event()
        self.pushed = False
        self.ln_done = torch.zeros(1, dtype=torch.int32, device=device)  # the LN kernel's CTA count
        self.n_rs = ops.fp8_gemm_ctas(M, D)
        self.flags_view = r[self.off["flags"]:self.off["flags"] + 4 * 8 * self.N_FLAG_SETS]
        self.bar = torch.zeros(1, dtype=torch.float32, device=device)
        self.ag_uses = self.rs_uses = self.ar_calls = 0
        self.key = key

    def begin_forward(self):
        """Start every forward from zeroed counters: zero this rank's counters,
        then a one-element all-reduce (on the stream, no host wait) as the
        barrier after which peers may signal again. Every signal of the previous
        forward was waited for by its receiver inside that forward, so none is
        lost; and the expected values of a forward are the same every time,
        which keeps a captured CUDA graph of it valid on replay."""
        self.flags_view.zero_()
        dist.all_reduce(self.bar, group=self.group)
        self.ag_uses = self.rs_uses = self.ar_calls = 0
        self.pushed = False   # the previous forward's pushes were joined at its end

    # ---- fused steps
    def gather_ln(self, x, eps, **ln):
        """LN-modulate-quant of this rank's rows into every rank's gather buffer
        (the next GEMM starts on the local rows and waits per remote shard).

        push "sm": one kernel stores the rows over NVLink and signals (row widths
        that are a multiple of 512, up to 4096). Otherwise, or with push "ce",
        the kernel writes this rank's own rows and the copy engines push them to
        every other rank on a side stream."""
        if self.push == "sm" and self.D % 512 == 0 and self.D <= 4096:
            ops.ln_mod_quant_tp(x, eps, q_rows=self.t_gq_rows, s_rows=self.t_gs_rows,
                                flags=self.t_flags[0], done=self.ln_done, rank=self.rank,
                                world=self.world, ldq=self.D, **ln)
            self.ag_uses += 1
            return
        main = torch.cuda.current_stream(x.device)
        if self.pushed:
            main.wait_event(self.ev_push)  # the previous push has read these rows
        r0, r1 = self.rank * self.Ml, (self.rank + 1) * self.Ml
        ops.ln_mod_quant(x, eps, q=self.gq[r0:r1], qscale=self.gs[r0:r1], **ln)
        self.ev_ln.record(main)
        self.side.wait_event(self.ev_ln)
        ops.tp_push(self.gq[r0:r1], self.t_gq_rows, self.gs[r0:r1], self.t_gs_rows,
                    flags=self.t_flags[0], rank=self.rank, world=self.world, stream=self.side)
        self.ev_push.record(self.side)
        self.pushed = True
        self.ag_uses += 1

    def rejoin(self, stream):
        """Make ``stream`` wait for the side stream's last push (push "ce")."""
        if self.pushed:
            stream.wait_event(self.ev_push)

    def tp_gemm(self, *, peer=False, v_ring=None):
        """TpGemm table for a GEMM that reads the gather buffer (waits per remote
        shard) or stores its partial into the owners' rs slots (peer=True).
        ``v_ring``: (ring, col0, frame_tokens, slot0, n_slots), columns [col0, N)
        of a gathered-input GEMM into the frame ring."""
        t = _lib.TpGemm()
        if v_ring is not None:
            ring, col0, ft, slot0, n_slots = v_ring
            t.v_ring = ctypes.pointer(_lib.VRing(ctypes.c_void_p(ring.data_ptr()), ring.stride(0),
                                                 int(col0), int(ft), int(slot0), int(n_slots)))
        t.rows_per_rank, t.rank, t.world = self.Ml, self.rank, self.world
        if peer:
            t.ag_flags = None
            for d in range(self.world):
                t.rs_slot[d] = self.rs_slot_addrs[d]
                t.rs_flags[d] = self.t_flags[1].p[d]
            t.ld_rs = self.D
            self.rs_uses += 1
        else:
            t.ag_flags = self.my_flags[0]
            t.ag_expected = self.ag_uses & 0xffffffff   # one push signal per use
        return t

    def rs_expected(self):
        return (self.rs_uses * self.n_rs) & 0xffffffff

    def allreduce(self, t, op, status=None):
        self.ar_calls += 1
        ops.tp_allreduce(t, op, slots=self.t_ar[self.ar_calls & 1], flags=self.t_flags[2],
                         rank=self.rank, world=self.world, epoch=self.ar_calls, status=status)

    def close(self):
        for b in self.peer_bases:
            ops.ipc_close(b)
        self.peer_bases = []


class _TPLayer:
    """One block's weights for rank r of P."""

    def __init__(self, sd, prefix, cfg: SRDiTConfig, device, rank, world):
        D, F = cfg.dim, cfg.ffn_dim
        Dl, Fl = D // world, F // world
        fs = slice(rank * Dl, (rank + 1) * Dl)
        ffs = slice(rank * Fl, (rank + 1) * Fl)
        g = lambda n: sd[f"{prefix}{n}"].to(device)  # noqa: E731
        bf = lambda n: g(n).to(torch.bfloat16).contiguous()  # noqa: E731

        def rowpar(name):
            # quantise per output channel over the full input width, then slice K
            wq, ws = quantize_weight(bf(name))
            cols = fs if wq.shape[1] == D else ffs
            return wq[:, cols].contiguous(), ws

        wqkv = torch.cat([g("self_attn.q.weight")[fs], g("self_attn.k.weight")[fs],
                          g("self_attn.v.weight")[fs]]).to(torch.bfloat16).contiguous()
        self.w_qkv, self.s_qkv = quantize_weight(wqkv)
        self.b_qkv = torch.cat([bf("self_attn.q.bias")[fs], bf("self_attn.k.bias")[fs],
                                bf("self_attn.v.bias")[fs]]).contiguous()
        self.w_o, self.s_o = rowpar("self_attn.o.weight")
        self.b_o = bf("self_attn.o.bias")
        self.nq = bf("self_attn.norm_q.weight")[fs].contiguous()
        self.nk = bf("self_attn.norm_k.weight")[fs].contiguous()
        self.w_cq, self.s_cq = quantize_weight(
            g("cross_attn.q.weight")[fs].to(torch.bfloat16).contiguous())
        self.b_cq = bf("cross_attn.q.bias")[fs].contiguous()
        wckv = torch.cat([g("cross_attn.k.weight")[fs], g("cross_attn.v.weight")[fs]])
        self.w_ckv, self.s_ckv = quantize_weight(wckv.to(torch.bfloat16).contiguous())
        self.b_ckv = torch.cat([bf("cross_attn.k.bias")[fs],
                                bf("cross_attn.v.bias")[fs]]).contiguous()
        self.w_co, self.s_co = rowpar("cross_attn.o.weight")
        self.b_co = bf("cross_attn.o.bias")
        self.cnq = bf("cross_attn.norm_q.weight")[fs].contiguous()
        self.cnk = bf("cross_attn.norm_k.weight")[fs].contiguous()
        self.n3w, self.n3b = bf("norm3.weight"), bf("norm3.bias")
        self.w_f0, self.s_f0 = quantize_weight(
            g("ffn.0.weight")[ffs].to(torch.bfloat16).contiguous())
        self.b_f0 = bf("ffn.0.bias")[ffs].contiguous()
        self.w_f2, self.s_f2 = rowpar("ffn.2.weight")
        self.b_f2 = bf("ffn.2.bias")
        self.modulation = g("modulation").float().reshape(6, D).contiguous()


class TPSRDiT(SRDiT):
    """``SRDiT`` with its blocks sharded over the ranks of ``comm``.

    Embeddings and the head are replicated: every rank computes them and
    returns the full refined latent. The K/V ring holds this rank's heads.
    """

    def __init__(self, cfg: SRDiTConfig, sd: dict, device="cuda", comm: TPComm | None = None,
                 fused: bool = True, local_scales: bool = True):
        """``fused``: collectives fused into the kernels over peer memory
        (``PeerComm``); False: the same sharding with library (NCCL) collectives.
        ``local_scales``: per-token e4m3 scales of the row-parallel inputs over this
        rank's slice (no all-reduce); False: over the full row (all-reduced max)."""
        self.local_scales = local_scales
        if comm is None:
            comm = PeerComm() if fused else TPComm()
        self.comm = comm
        self.fused = isinstance(comm, PeerComm)
        P = self.comm.world
        if cfg.num_heads % P or cfg.ffn_dim % P:
            raise _lib.SrditError(f"{P} ranks must divide the {cfg.num_heads} heads and the "
                                  f"FFN width {cfg.ffn_dim}")
        self.rank, self.world = self.comm.rank, P
        super().__init__(cfg, sd, device)

    def _make_layer(self, sd, prefix):
        return _TPLayer(sd, prefix, self.cfg, self.device, self.rank, self.world)

    @property
    def kv_width(self):
        return self.cfg.dim // self.world

    def _text_kv(self, ly, ctxq, ctxs, ckv):
        """This rank's heads of the text K | V; norm_k over the full width needs
        the all-reduced sum of squares (a library all-reduce: once per context)."""
        c = self.cfg
        Dl = self.kv_width
        self.ops.fp8_gemm(ctxq, ctxs, ly.w_ckv, ly.s_ckv, ly.b_ckv, ckv)
        ss = self.ops.row_reduce(ckv[:, :Dl], "sumsq")
        self.comm.all_reduce_sum(ss)
        self.ops.rms_rope(ckv[:, :Dl], ly.cnk, c.eps, ckv[:, :Dl], frame_tokens=ckv.shape[0],
                          ss=ss, norm_width=c.dim)

    # ------------------------------------------------------------------ forward
    def forward_chunk(self, latent, t, context, *, cache=None, t_offset=0, update_cache=False,
                      anchor_kv=None, anchor_align="frame", return_kv=False, ctx_emb=None,
                      text=None, kv_only=False, independent_frames=False):
        """``SRDiT.forward_chunk`` on this rank's shard; same arguments and result
        (``anchor_kv`` / the returned K/V hold this rank's heads)."""
        if kv_only and (return_kv or not update_cache):
            raise _lib.SrditError("kv_only is for a cache-refresh forward (update_cache=True, "
                                  "no return_kv)")
        if self.fused:
            return self._forward_fused(latent, t, context, cache=cache, t_offset=t_offset,
                                       update_cache=update_cache, anchor_kv=anchor_kv,
                                       anchor_align=anchor_align, return_kv=return_kv,
                                       ctx_emb=ctx_emb, text=text, kv_only=kv_only,
                                       independent_frames=independent_frames)
        c = self.cfg
        ops = self.ops
        if not self.graph_capture:
            self.set_t_offset(t_offset)
        P, r = self.world, self.rank
        comm = self.comm
        D, Dl, Fl = c.dim, c.dim // P, c.ffn_dim // P
        Hl = c.num_heads // P
        if text is not None:
            ctx_emb = text.ctx_emb
        S = self._setup(latent, t, context, cache, anchor_kv, anchor_align, ctx_emb, Hl, Dl,
                        independent_frames)
        x_full, e0, e, ctx, grid, cache = S.x, S.e0, S.e, S.ctx, S.grid, S.cache
        f, h, w = grid
        L, M, Lc = S.L, S.M, S.Lc
        if M % P:
            raise _lib.SrditError(f"{M} tokens do not split over {P} ranks")
        Ml = M // P
        x = x_full[r * Ml:(r + 1) * Ml].contiguous()
        dev = self.device
        bf16, f32, f8 = torch.bfloat16, torch.float32, torch.float8_e4m3fn
        b = self._buf
        xq_l, xs_l = b("tp_xq_l", (Ml, D), f8), b("tp_xs_l", (Ml,), f32)
        xq, xs = b("tp_xq", (M, D), f8), b("tp_xs", (M,), f32)
        qkv = b("tp_qkv", (M, 3 * Dl), bf16)
        qb = b("tp_q", (M, Dl), bf16)
        att = b("tp_att", (M, Dl), bf16)
        aq, as_ = b("tp_aq", (M, Dl), f8), b("tp_as", (M,), f32)
        part = b("tp_part", (M, D), bf16)
        y_l = b("tp_y", (Ml, D), bf16)
        ss = b("tp_ss", (2 * M,), f32)
        ssc = b("tp_ssc", (M + Lc,), f32)
        am = b("tp_am", (M,), f32)
        hbuf = b("tp_h", (M, Fl), bf16)
        hq, hs = b("tp_hq", (M, Fl), f8), b("tp_hs", (M,), f32)
        ckv = b("tp_ckv", (Lc, 2 * Dl), bf16)
        ctxq, ctxs = ops.quant_rowwise(ctx) if text is None else (None, None)
        mods = torch.stack([ly.modulation for ly in self.layers]) + e0[None]
        kv_out = [] if return_kv else None
        st = self.status
        cos, sin = self.rope_cos, self.rope_sin
        slot_cur = S.slot_cur
        v_direct = L % 32 == 0 and Dl % 64 == 0   # the GEMM can store V into ring slots

        def gather_quantised():
            comm.all_gather(xq, xq_l)
            comm.all_gather(xs, xs_l)

        def rowpar_residual(a_bf16, w_q, w_s, bias, gate):
            if self.local_scales:   # per-token scale over this rank's slice
                ops.quant_rowwise(a_bf16, q=aq, scale=as_)
            else:                   # over the full row: all-reduce the slices' max |a|
                ops.row_reduce(a_bf16, "absmax", out=am)
                comm.all_reduce_max(am)
                ops.quant_rowwise(a_bf16, amax=am, q=aq, scale=as_)
            ops.fp8_gemm(aq, as_, w_q, w_s, None, part)          # bf16(acc * sa * sb)
            comm.reduce_scatter(y_l, part)
            ops.residual(x, y_l, bias=bias, gate=gate)

        for li, ly in enumerate(self.layers):
            em = mods[li]
            kr, vr = cache.k[li], cache.v[li]
            # --- self attention
            ops.ln_mod_quant(x, c.eps, shift=em[0], scale=em[1], q=xq_l, qscale=xs_l)
            gather_quantised()
            vcopy = {} if v_direct else dict(v_src=qkv[:, 2 * Dl:], v_dst=vr)
            if kv_only and li == len(self.layers) - 1:
                # the refresh pass's last block: its K / V into the ring, nothing else
                ops.fp8_gemm(xq, xs, ly.w_qkv[Dl:], ly.s_qkv[Dl:], ly.b_qkv[Dl:], qkv[:, Dl:],
                             v_ring=(vr, Dl, L, slot_cur, cache.cap) if v_direct else None)
                ops.row_reduce(qkv[:, Dl:2 * Dl], "sumsq", out=ss[M:])
                comm.all_reduce_sum(ss[M:])
                ops.rms_rope(qkv[:, Dl:2 * Dl], ly.nk, c.eps, kr, frame_tokens=L,
                             slot0=slot_cur, n_slots=cache.cap, cos=cos, sin=sin, grid_h=h,
                             grid_w=w, t_offset_dev=self.t_offset_dev, ss=ss[M:], norm_width=D,
                             **vcopy)
                break
            # V goes straight into its ring slot (else the K kernel copies it there)
            ops.fp8_gemm(xq, xs, ly.w_qkv, ly.s_qkv, ly.b_qkv, qkv,
                         v_ring=(vr, 2 * Dl, L, slot_cur, cache.cap) if v_direct else None)
            ops.row_reduce(qkv[:, :Dl], "sumsq", out=ss[:M])
            ops.row_reduce(qkv[:, Dl:2 * Dl], "sumsq", out=ss[M:])
            comm.all_reduce_sum(ss)
            ops.rms_rope(qkv[:, :Dl], ly.nq, c.eps, qb, frame_tokens=L, cos=cos, sin=sin,
                         grid_h=h, grid_w=w, t_offset_dev=self.t_offset_dev, ss=ss[:M],
                         norm_width=D)
            ops.rms_rope(qkv[:, Dl:2 * Dl], ly.nk, c.eps, kr, frame_tokens=L, slot0=slot_cur,
                         n_slots=cache.cap, cos=cos, sin=sin, grid_h=h, grid_w=w,
                         t_offset_dev=self.t_offset_dev, ss=ss[M:], norm_width=D, **vcopy)
            ak = av = None
            if anchor_kv is not None:
                ak, av = anchor_kv[li]
            ops.winattn(qb, kr, vr, att, params_dev=S.params_dev, n_w=S.n_w,
                        p_stride=int(S.plan["p_stride"]), anchor_mode=S.amode, geom=S.geom,
                        tiling=S.tiling, k_anchor=ak, v_anchor=av, status=st, flops=S.flops)
            if return_kv:
                idx = (torch.arange(f, device=dev) + slot_cur) % cache.cap
                kv_out.append((kr.view(cache.cap, L, Dl)[idx].reshape(M, Dl).clone(),
                               vr.view(cache.cap, L, Dl)[idx].reshape(M, Dl).clone()))
            rowpar_residual(att, ly.w_o, ly.s_o, ly.b_o, em[2])
            # --- cross attention
            ops.ln_mod_quant(x, c.eps, ln_weight=ly.n3w, ln_bias=ly.n3b, q=xq_l, qscale=xs_l)
            gather_quantised()
            ops.fp8_gemm(xq, xs, ly.w_cq, ly.s_cq, ly.b_cq, qb)
            ops.row_reduce(qb, "sumsq", out=ssc[:M])
            if text is None:
                ops.fp8_gemm(ctxq, ctxs, ly.w_ckv, ly.s_ckv, ly.b_ckv, ckv)
                ops.row_reduce(ckv[:, :Dl], "sumsq", out=ssc[M:])
                comm.all_reduce_sum(ssc)
                ops.rms_rope(ckv[:, :Dl], ly.cnk, c.eps, ckv[:, :Dl], frame_tokens=Lc,
                             ss=ssc[M:], norm_width=D)
            else:
                comm.all_reduce_sum(ssc[:M])
                ckv = text.kv[li]
            ops.rms_rope(qb, ly.cnq, c.eps, qb, frame_tokens=M, ss=ssc[:M], norm_width=D)
            ops.winattn(qb, ckv[:, :Dl], ckv[:, Dl:], att, params_dev=S.cp_params,
                        n_w=S.cp_nw, p_stride=19, anchor_mode=0, geom=S.cgeom,
                        tiling=S.cp_tiling, status=st, flops=S.cross_flops)
            rowpar_residual(att, ly.w_co, ly.s_co, ly.b_co, None)
            # --- FFN
            ops.ln_mod_quant(x, c.eps, shift=em[3], scale=em[4], q=xq_l, qscale=xs_l)
            gather_quantised()
            am.zero_()
            ops.fp8_gemm(xq, xs, ly.w_f0, ly.s_f0, ly.b_f0, hbuf, epilogue="gelu", row_amax=am)
            if not self.local_scales:
                comm.all_reduce_max(am)
            ops.quant_rowwise(hbuf, amax=am, q=hq, scale=hs)
            ops.fp8_gemm(hq, hs, ly.w_f2, ly.s_f2, None, part)
            comm.reduce_scatter(y_l, part)
            ops.residual(x, y_l, bias=ly.b_f2, gate=em[5])
        if update_cache:
            cache.commit(f)
        if kv_only:
            return None
        xg = b("tp_xg", (M, D), bf16)
        comm.all_gather(xg, x)
        out = self.head(xg, e, grid)
        return (out, kv_out) if return_kv else out

    def _forward_fused(self, latent, t, context, *, cache, t_offset, update_cache, anchor_kv,
                       anchor_align, return_kv, ctx_emb, text=None, kv_only=False,
                       independent_frames=False):
        """The sharded block with its collectives fused into the kernels: each
        rank's LN-quant rows are pushed by the copy engines into every rank's
        gather buffer and the next GEMM waits per remote shard (all-gather);
        row-parallel GEMMs store their bf16 partials into the owners' receive
        slots tile by tile and the owner's residual kernel waits and sums
        (reduce-scatter); per-token statistics go through the one-block peer
        all-reduce."""
        c = self.cfg
        ops = self.ops
        if not self.graph_capture:
            self.set_t_offset(t_offset)
        P, r = self.world, self.rank
        comm = self.comm
        D, Dl, Fl = c.dim, c.dim // P, c.ffn_dim // P
        Hl = c.num_heads // P
        if text is not None:
            ctx_emb = text.ctx_emb
        S = self._setup(latent, t, context, cache, anchor_kv, anchor_align, ctx_emb, Hl, Dl,
                        independent_frames)
        x_full, e0, e, ctx, grid, cache = S.x, S.e0, S.e, S.ctx, S.grid, S.cache
        f, h, w = grid
        L, M, Lc = S.L, S.M, S.Lc
        comm.setup(M, D, self.device)
        comm.begin_forward()
        Ml = comm.Ml
        x = x_full[r * Ml:(r + 1) * Ml].contiguous()
        dev = self.device
        bf16, f32, f8 = torch.bfloat16, torch.float32, torch.float8_e4m3fn
        b = self._buf
        xq, xs = comm.gq, comm.gs
        qkv = b("tp_qkv", (M, 3 * Dl), bf16)
        qb = b("tp_q", (M, Dl), bf16)
        att = b("tp_att", (M, Dl), bf16)
        aq, as_ = b("tp_aq", (M, Dl), f8), b("tp_as", (M,), f32)
        ss = b("tp_ss", (2 * M,), f32)
        ssc = b("tp_ssc", (M + Lc,), f32)
        am = b("tp_am", (M,), f32)
        hbuf = b("tp_h", (M, Fl), bf16)
        hq, hs = b("tp_hq", (M, Fl), f8), b("tp_hs", (M,), f32)
        ckv = b("tp_ckv", (Lc, 2 * Dl), bf16)
        ctxq, ctxs = ops.quant_rowwise(ctx) if text is None else (None, None)
        mods = torch.stack([ly.modulation for ly in self.layers]) + e0[None]
        kv_out = [] if return_kv else None
        st = self.status
        cos, sin = self.rope_cos, self.rope_sin
        slot_cur = S.slot_cur
        v_direct = L % 32 == 0 and Dl % 64 == 0   # the GEMM can store V into ring slots
        rs_flags = comm.my_flags[1]

        def rowpar_residual(a_bf16, w_q, w_s, bias, gate):
            if self.local_scales:   # per-token scale over this rank's slice
                ops.quant_rowwise(a_bf16, q=aq, scale=as_)
            else:
                ops.row_reduce(a_bf16, "absmax", out=am)
                comm.allreduce(am, "max", st)
                ops.quant_rowwise(a_bf16, amax=am, q=aq, scale=as_)
            ops.fp8_gemm_tp(aq, as_, w_q, w_s, None, None, tp=comm.tp_gemm(peer=True),
                            epilogue="peer", status=st)
            ops.residual_tp(x, comm.rs, bias=bias, gate=gate, flags=rs_flags,
                            expected=comm.rs_expected(), status=st)

        for li, ly in enumerate(self.layers):
            em = mods[li]
            kr, vr = cache.k[li], cache.v[li]
            # --- self attention
            comm.gather_ln(x, c.eps, shift=em[0], scale=em[1])
            vcopy = {} if v_direct else dict(v_src=qkv[:, 2 * Dl:], v_dst=vr)
            if kv_only and li == len(self.layers) - 1:
                # the refresh pass's last block: its K / V into the ring, nothing else
                vring = (vr, Dl, L, slot_cur, cache.cap) if v_direct else None
                ops.fp8_gemm_tp(xq, xs, ly.w_qkv[Dl:], ly.s_qkv[Dl:], ly.b_qkv[Dl:],
                                qkv[:, Dl:], status=st, tp=comm.tp_gemm(v_ring=vring))
                ops.row_reduce(qkv[:, Dl:2 * Dl], "sumsq", out=ss[M:])
                comm.allreduce(ss[M:], "sum", st)
                ops.rms_rope(qkv[:, Dl:2 * Dl], ly.nk, c.eps, kr, frame_tokens=L,
                             slot0=slot_cur, n_slots=cache.cap, cos=cos, sin=sin, grid_h=h,
                             grid_w=w, t_offset_dev=self.t_offset_dev, ss=ss[M:], norm_width=D,
                             **vcopy)
                break
            # V goes straight into its ring slot (else the K kernel copies it there)
            ops.fp8_gemm_tp(xq, xs, ly.w_qkv, ly.s_qkv, ly.b_qkv, qkv, status=st, tp=comm.tp_gemm(
                v_ring=(vr, 2 * Dl, L, slot_cur, cache.cap) if v_direct else None))
            ops.row_reduce(qkv[:, :Dl], "sumsq", out=ss[:M])
            ops.row_reduce(qkv[:, Dl:2 * Dl], "sumsq", out=ss[M:])
            comm.allreduce(ss, "sum", st)
            ops.rms_rope(qkv[:, :Dl], ly.nq, c.eps, qb, frame_tokens=L, cos=cos, sin=sin,
                         grid_h=h, grid_w=w, t_offset_dev=self.t_offset_dev, ss=ss[:M],
                         norm_width=D)
            ops.rms_rope(qkv[:, Dl:2 * Dl], ly.nk, c.eps, kr, frame_tokens=L, slot0=slot_cur,
                         n_slots=cache.cap, cos=cos, sin=sin, grid_h=h, grid_w=w,
                         t_offset_dev=self.t_offset_dev, ss=ss[M:], norm_width=D, **vcopy)
            ak = av = None
            if anchor_kv is not None:
                ak, av = anchor_kv[li]
            ops.winattn(qb, kr, vr, att, params_dev=S.params_dev, n_w=S.n_w,
                        p_stride=int(S.plan["p_stride"]), anchor_mode=S.amode, geom=S.geom,
                        tiling=S.tiling, k_anchor=ak, v_anchor=av, status=st, flops=S.flops)
            if return_kv:
                idx = (torch.arange(f, device=dev) + slot_cur) % cache.cap
                kv_out.append((kr.view(cache.cap, L, Dl)[idx].reshape(M, Dl).clone(),
                               vr.view(cache.cap, L, Dl)[idx].reshape(M, Dl).clone()))
            rowpar_residual(att, ly.w_o, ly.s_o, ly.b_o, em[2])
            # --- cross attention
            comm.gather_ln(x, c.eps, ln_weight=ly.n3w, ln_bias=ly.n3b)
            ops.fp8_gemm_tp(xq, xs, ly.w_cq, ly.s_cq, ly.b_cq, qb, tp=comm.tp_gemm(), status=st)
            ops.row_reduce(qb, "sumsq", out=ssc[:M])
            if text is None:
                ops.fp8_gemm(ctxq, ctxs, ly.w_ckv, ly.s_ckv, ly.b_ckv, ckv)
                ops.row_reduce(ckv[:, :Dl], "sumsq", out=ssc[M:])
                comm.allreduce(ssc, "sum", st)
                ops.rms_rope(ckv[:, :Dl], ly.cnk, c.eps, ckv[:, :Dl], frame_tokens=Lc,
                             ss=ssc[M:], norm_width=D)
            else:
                comm.allreduce(ssc[:M], "sum", st)
                ckv = text.kv[li]
            ops.rms_rope(qb, ly.cnq, c.eps, qb, frame_tokens=M, ss=ssc[:M], norm_width=D)
            ops.winattn(qb, ckv[:, :Dl], ckv[:, Dl:], att, params_dev=S.cp_params,
                        n_w=S.cp_nw, p_stride=19, anchor_mode=0, geom=S.cgeom,
                        tiling=S.cp_tiling, status=st, flops=S.cross_flops)
            rowpar_residual(att, ly.w_co, ly.s_co, ly.b_co, None)
            # --- FFN
            comm.gather_ln(x, c.eps, shift=em[3], scale=em[4])
            am.zero_()
            ops.fp8_gemm_tp(xq, xs, ly.w_f0, ly.s_f0, ly.b_f0, hbuf, tp=comm.tp_gemm(),
                            epilogue="gelu", row_amax=am, status=st)
            if not self.local_scales:
                comm.allreduce(am, "max", st)
            ops.quant_rowwise(hbuf, amax=am, q=hq, scale=hs)
            ops.fp8_gemm_tp(hq, hs, ly.w_f2, ly.s_f2, None, None, tp=comm.tp_gemm(peer=True),
                            epilogue="peer", status=st)
            ops.residual_tp(x, comm.rs, bias=ly.b_f2, gate=em[5], flags=rs_flags,
                            expected=comm.rs_expected(), status=st)
        if update_cache:
            cache.commit(f)
        comm.rejoin(torch.cuda.current_stream(dev))   # a side stream's pushes rejoin
        if kv_only:
            return None
        xg = b("tp_xg", (M, D), bf16)
        comm.all_gather(xg, x)
        out = self.head(xg, e, grid)
        return (out, kv_out) if return_kv else out
