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
The per-token activation scales are the full-row ones (all-reduced amax), so
each partial product is the TP=1 product restricted to a K slice; what
differs from one GPU is the fp32 summation order and the bf16 rounding of
each rank's partial before the sum.

Collectives go through ``TPComm`` (NCCL via torch.distributed). Every rank
issues the same collectives in the same order.
"""
from __future__ import annotations

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

    def __init__(self, cfg: SRDiTConfig, sd: dict, device="cuda", comm: TPComm | None = None):
        self.comm = comm if comm is not None else TPComm()
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

    # ------------------------------------------------------------------ forward
    def forward_chunk(self, latent, t, context, *, cache=None, t_offset=0, update_cache=False,
                      anchor_kv=None, anchor_align="frame", return_kv=False, ctx_emb=None):
        """``SRDiT.forward_chunk`` on this rank's shard; same arguments and result
        (``anchor_kv`` / the returned K/V hold this rank's heads)."""
        c = self.cfg
        P, r = self.world, self.rank
        comm = self.comm
        D, Dl, Fl = c.dim, c.dim // P, c.ffn_dim // P
        Hl = c.num_heads // P
        S = self._setup(latent, t, context, cache, anchor_kv, anchor_align, ctx_emb, Hl, Dl)
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
        ctxq, ctxs = ops.quant_rowwise(ctx)
        mods = torch.stack([ly.modulation for ly in self.layers]) + e0[None]
        kv_out = [] if return_kv else None
        st = self.status
        cos, sin = self.rope_cos, self.rope_sin
        slot_cur = S.slot_cur

        def gather_quantised():
            comm.all_gather(xq, xq_l)
            comm.all_gather(xs, xs_l)

        def rowpar_residual(a_bf16, w_q, w_s, bias, gate):
            # per-token scale over the full row: all-reduce the slices' max |a|
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
            ops.fp8_gemm(xq, xs, ly.w_qkv, ly.s_qkv, ly.b_qkv, qkv)
            ops.row_reduce(qkv[:, :Dl], "sumsq", out=ss[:M])
            ops.row_reduce(qkv[:, Dl:2 * Dl], "sumsq", out=ss[M:])
            comm.all_reduce_sum(ss)
            ops.rms_rope(qkv[:, :Dl], ly.nq, c.eps, qb, frame_tokens=L, cos=cos, sin=sin,
                         grid_h=h, grid_w=w, t_offset=t_offset, ss=ss[:M], norm_width=D)
            ops.rms_rope(qkv[:, Dl:2 * Dl], ly.nk, c.eps, kr, frame_tokens=L, slot0=slot_cur,
                         n_slots=cache.cap, cos=cos, sin=sin, grid_h=h, grid_w=w,
                         t_offset=t_offset, v_src=qkv[:, 2 * Dl:], v_dst=vr, ss=ss[M:],
                         norm_width=D)
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
            ops.fp8_gemm(ctxq, ctxs, ly.w_ckv, ly.s_ckv, ly.b_ckv, ckv)
            ops.row_reduce(qb, "sumsq", out=ssc[:M])
            ops.row_reduce(ckv[:, :Dl], "sumsq", out=ssc[M:])
            comm.all_reduce_sum(ssc)
            ops.rms_rope(qb, ly.cnq, c.eps, qb, frame_tokens=M, ss=ssc[:M], norm_width=D)
            ops.rms_rope(ckv[:, :Dl], ly.cnk, c.eps, ckv[:, :Dl], frame_tokens=Lc,
                         ss=ssc[M:], norm_width=D)
            ops.winattn(qb, ckv[:, :Dl], ckv[:, Dl:], att, params_dev=S.cp_params,
                        n_w=S.cp_nw, p_stride=19, anchor_mode=0, geom=S.cgeom,
                        tiling=S.cp_tiling, status=st, flops=S.cross_flops)
            rowpar_residual(att, ly.w_co, ly.s_co, ly.b_co, None)
            # --- FFN
            ops.ln_mod_quant(x, c.eps, shift=em[3], scale=em[4], q=xq_l, qscale=xs_l)
            gather_quantised()
            am.zero_()
            ops.fp8_gemm(xq, xs, ly.w_f0, ly.s_f0, ly.b_f0, hbuf, epilogue="gelu", row_amax=am)
            comm.all_reduce_max(am)
            ops.quant_rowwise(hbuf, amax=am, q=hq, scale=hs)
            ops.fp8_gemm(hq, hs, ly.w_f2, ly.s_f2, None, part)
            comm.reduce_scatter(y_l, part)
            ops.residual(x, y_l, bias=ly.b_f2, gate=em[5])
        if update_cache:
            cache.commit(f)
        xg = b("tp_xg", (M, D), bf16)
        comm.all_gather(xg, x)
        out = self.head(xg, e, grid)
        return (out, kv_out) if return_kv else out
