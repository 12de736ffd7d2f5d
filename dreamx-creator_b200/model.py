"""SR-DiT 5B streaming forward on the B200 kernels.

The module tree and parameter names follow the reference's ``WanModel``
(video_refiner/wan/modules/sr_dit/models.py:1390-1633): ``patch_embedding``,
``text_embedding.{0,2}``, ``time_embedding.{0,2}``, ``time_projection.1``,
``blocks.{i}.{norm3, self_attn.{q,k,v,o,norm_q,norm_k}, cross_attn.{...},
ffn.{0,2}, modulation}``, ``head.{head, modulation}``, so a reference state dict
loads 1:1 (``SRDiT.from_state_dict``).

One call of ``SRDiT.forward_chunk`` is the reference's ``_forward_inference``
(models.py:1877-2002) for one sample: embeddings, 30 blocks, head, unpatchify.
Per block the work is 10 launches of libsrdit_b200.so kernels, in this order:

  ln_mod_quant(x; e0, e1)            -> x_q            norm1 + modulate + quantise
  fp8_gemm(x_q, W_qkv)               -> qkv            self q|k|v (fused N = 3*dim)
  rms_rope(q) ; rms_rope(k, +v)      -> q, K/V ring    norm_q/norm_k, 3-D RoPE, cache write
  winattn(q, K/V ring [, anchor])    -> a              block-grid window attention
  quant_rowwise(a)                   -> a_q
  fp8_gemm(a_q, W_o, gated_res e2)   -> x              x + o(a) * e2
  ln_mod_quant(x; norm3 affine)      -> x_q
  fp8_gemm(x_q, W_cq) ; rms          -> qc             cross q + norm_q
  winattn(qc, text K/V)              -> c              cross attention (dense window)
  quant_rowwise(c) ; fp8_gemm(res)   -> x              x + cross_o(c)
  ln_mod_quant(x; e3, e4)            -> x_q
  fp8_gemm(x_q, W_ffn0, gelu+amax)   -> h, amax        ffn.0 + GELU(tanh) + row amax
  quant_rowwise(h, amax)             -> h_q
  fp8_gemm(h_q, W_ffn2, gated_res e5)-> x              x + ffn.2(h) * e5

The per-layer text K/V (cross_attn.k/v over the 512 text tokens) comes from
``SRDiT.text_cache``: the same GEMM + RMSNorm kernels run once per text context
(the reference recomputes them in every forward, models.py:1048-1054; the
values do not change within a clip). A forward given no cache computes them
inline.

The KV cache is a per-layer ring of ``kv_len + chunk`` frame slots: the current
chunk's roped K and V are written straight into their slots by ``rms_rope`` and
the window kernel reads the cached frames in place, so no ``torch.cat`` copy or
truncation happens (the reference concatenates and slices per layer,
attention.py:1506-1510, :964-974).

The embeddings (patch Conv3d, text MLP, time MLP) and the output head run once
per forward outside the block loop and stay in torch, with the reference's
dtypes (bf16 embeddings; fp32 time MLP and head, as under its CUDA fp32
autocast, models.py:1845-1849, :1380-1383).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, blockgrid, ops
from .fp8_linear import quantize_weight


@dataclass
class SRDiTConfig:
    dim: int = 3072
    ffn_dim: int = 14336
    num_heads: int = 24
    num_layers: int = 30
    in_dim: int = 48
    out_dim: int = 48
    text_dim: int = 4096
    freq_dim: int = 256
    text_len: int = 512
    patch_size: tuple = (1, 2, 2)
    eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_rows: int = 1024
    # window attention
    block_t: int = 3
    block_hw: tuple = (8, 8)
    block_radius_hw: tuple = (0, 0)
    block_radius_t: int | None = None
    kv_len: int = 9
    chunk_frames: int = 3


def sinusoidal_embedding_1d(dim, position):
    """models.py:66-77 (fp64)."""
    half = dim // 2
    position = position.to(torch.float64)
    sinusoid = torch.outer(position, torch.pow(10000, -torch.arange(half, device=position.device)
                                                .to(position).div(half)))
    return torch.cat([torch.cos(sinusoid), torch.sin(sinusoid)], dim=1)


def rope_tables(head_dim, rows, theta, device):
    """cos/sin (fp64 [rows, head_dim/2]) of WanModel._build_rope_freqs (models.py:1724-1737)."""
    t = head_dim - 4 * (head_dim // 6)
    s = 2 * (head_dim // 6)
    cols = []
    for d in (t, s, s):
        inv = 1.0 / torch.pow(theta, torch.arange(0, d, 2, dtype=torch.float64) / d)
        ang = torch.outer(torch.arange(rows, dtype=torch.float64), inv)
        cols.append(torch.polar(torch.ones_like(ang), ang))
    f = torch.cat(cols, dim=1)
    return f.real.contiguous().to(device), f.imag.contiguous().to(device)


class _Layer:
    """Prepared per-block weights (fp8 + scales, bf16 biases/norms, fp32 modulation)."""

    def __init__(self, sd, prefix, cfg, device):
        g = lambda n: sd[f"{prefix}{n}"].to(device)  # noqa: E731
        bf = lambda n: g(n).to(torch.bfloat16).contiguous()  # noqa: E731
        D = cfg.dim
        wqkv = torch.cat([g("self_attn.q.weight"), g("self_attn.k.weight"),
                          g("self_attn.v.weight")]).to(torch.bfloat16)
        self.w_qkv, self.s_qkv = quantize_weight(wqkv)
        self.b_qkv = torch.cat([bf("self_attn.q.bias"), bf("self_attn.k.bias"),
                                bf("self_attn.v.bias")]).contiguous()
        self.w_o, self.s_o = quantize_weight(bf("self_attn.o.weight"))
        self.b_o = bf("self_attn.o.bias")
        self.nq, self.nk = bf("self_attn.norm_q.weight"), bf("self_attn.norm_k.weight")
        self.w_cq, self.s_cq = quantize_weight(bf("cross_attn.q.weight"))
        self.b_cq = bf("cross_attn.q.bias")
        wckv = torch.cat([g("cross_attn.k.weight"), g("cross_attn.v.weight")]).to(torch.bfloat16)
        self.w_ckv, self.s_ckv = quantize_weight(wckv)
        self.b_ckv = torch.cat([bf("cross_attn.k.bias"), bf("cross_attn.v.bias")]).contiguous()
        self.w_co, self.s_co = quantize_weight(bf("cross_attn.o.weight"))
        self.b_co = bf("cross_attn.o.bias")
        self.cnq, self.cnk = bf("cross_attn.norm_q.weight"), bf("cross_attn.norm_k.weight")
        self.n3w, self.n3b = bf("norm3.weight"), bf("norm3.bias")
        self.w_f0, self.s_f0 = quantize_weight(bf("ffn.0.weight"))
        self.b_f0 = bf("ffn.0.bias")
        self.w_f2, self.s_f2 = quantize_weight(bf("ffn.2.weight"))
        self.b_f2 = bf("ffn.2.bias")
        self.modulation = g("modulation").float().reshape(6, D).contiguous()


class KVRing:
    """Per-layer K/V frame rings: ``cap = kv_len + chunk`` slots of one frame each."""

    def __init__(self, layers, frame_tokens, dim, kv_len, chunk, device):
        self.cap = kv_len + chunk
        self.kv_len = kv_len
        self.frame_tokens = frame_tokens
        self.k = [torch.zeros(self.cap * frame_tokens, dim, dtype=torch.bfloat16, device=device)
                  for _ in range(layers)]
        self.v = [torch.zeros_like(t) for t in self.k]
        self.start = 0      # slot of the oldest cached frame
        self.frames = 0     # cached frames (<= kv_len)

    def commit(self, f_cur):
        """After a cache-refresh forward: keep the newest kv_len frames."""
        total = self.frames + f_cur
        drop = max(0, total - self.kv_len)
        self.start = (self.start + drop) % self.cap
        self.frames = total - drop

    def reset(self):
        self.start = 0
        self.frames = 0


@dataclass
class TextCache:
    """Text embedding [Lc, D] and per-block cross-attention K | V [Lc, 2 * width]."""
    ctx_emb: torch.Tensor
    kv: list


class SRDiT:
    """The refiner transformer on the B200 kernels (inference only).

    ``ops`` is the table of kernel launchers the forward calls (the
    libsrdit_b200.so wrappers). A test may substitute a table of its own on a
    subclass to exercise the host-side orchestration without a GPU; the model
    itself has no other compute path and refuses to build without CUDA.
    """

    ops = ops
    require_cuda = True

    def __init__(self, cfg: SRDiTConfig, sd: dict, device="cuda"):
        if self.require_cuda and not torch.cuda.is_available():
            raise _lib.SrditError("SRDiT needs a CUDA device (there is no CPU path)")
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        D = cfg.dim
        self.head_dim = D // cfg.num_heads
        if self.head_dim != 128:
            raise _lib.SrditError("the B200 attention kernel needs head_dim 128")
        bf = lambda n: sd[n].to(dev, torch.bfloat16)  # noqa: E731
        f32 = lambda n: sd[n].to(dev, torch.float32)  # noqa: E731
        self.patch_w, self.patch_b = bf("patch_embedding.weight"), bf("patch_embedding.bias")
        self.txt = [(bf("text_embedding.0.weight"), bf("text_embedding.0.bias")),
                    (bf("text_embedding.2.weight"), bf("text_embedding.2.bias"))]
        self.tim = [(f32("time_embedding.0.weight"), f32("time_embedding.0.bias")),
                    (f32("time_embedding.2.weight"), f32("time_embedding.2.bias"))]
        self.tproj = (f32("time_projection.1.weight"), f32("time_projection.1.bias"))
        self.head_w, self.head_b = f32("head.head.weight"), f32("head.head.bias")
        self.head_mod = f32("head.modulation").reshape(2, D)
        self.layers = []
        for i in range(cfg.num_layers):
            self.layers.append(self._make_layer(sd, f"blocks.{i}."))
        self.rope_cos, self.rope_sin = rope_tables(self.head_dim, cfg.rope_rows, cfg.rope_theta, dev)
        self._bufs = {}
        self._cross_plans = {}
        self._temb = {}
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.t_offset_dev = torch.zeros(1, dtype=torch.int32, device=dev)
        # True while a caller captures forwards into a CUDA graph: the caller then
        # sets t_offset_dev itself before every replay
        self.graph_capture = False
        # width position of the token grid's column 0: 0, or a strip's first
        # column when this process refines one strip of a wider grid
        self.rope_w0 = 0

    # ------------------------------------------------------------------ construction
    @staticmethod
    def param_shapes(cfg: SRDiTConfig):
        D, F, C = cfg.dim, cfg.ffn_dim, cfg.in_dim
        p = math.prod(cfg.patch_size)
        shapes = {
            "patch_embedding.weight": (D, C, *cfg.patch_size), "patch_embedding.bias": (D,),
            "text_embedding.0.weight": (D, cfg.text_dim), "text_embedding.0.bias": (D,),
            "text_embedding.2.weight": (D, D), "text_embedding.2.bias": (D,),
            "time_embedding.0.weight": (D, cfg.freq_dim), "time_embedding.0.bias": (D,),
            "time_embedding.2.weight": (D, D), "time_embedding.2.bias": (D,),
            "time_projection.1.weight": (6 * D, D), "time_projection.1.bias": (6 * D,),
            "head.head.weight": (cfg.out_dim * p, D), "head.head.bias": (cfg.out_dim * p,),
            "head.modulation": (1, 2, D),
        }
        for i in range(cfg.num_layers):
            b = f"blocks.{i}."
            for m in ("self_attn", "cross_attn"):
                for n in ("q", "k", "v", "o"):
                    shapes[f"{b}{m}.{n}.weight"] = (D, D)
                    shapes[f"{b}{m}.{n}.bias"] = (D,)
                shapes[f"{b}{m}.norm_q.weight"] = (D,)
                shapes[f"{b}{m}.norm_k.weight"] = (D,)
            shapes[f"{b}norm3.weight"] = (D,)
            shapes[f"{b}norm3.bias"] = (D,)
            shapes[f"{b}ffn.0.weight"] = (F, D)
            shapes[f"{b}ffn.0.bias"] = (F,)
            shapes[f"{b}ffn.2.weight"] = (D, F)
            shapes[f"{b}ffn.2.bias"] = (D,)
            shapes[f"{b}modulation"] = (1, 6, D)
        return shapes

    @staticmethod
    def seeded_state_dict(cfg: SRDiTConfig, device="cuda", seed=0):
        """Seeded random weights of the reference architecture, generated on the
        device on first access, one tensor at a time (the 5B model never exists
        in bf16 at once). Each tensor has its own generator seeded from (seed,
        name), so its values do not depend on the order tensors are read in --
        a tensor-parallel rank slicing them gets exactly the full model's values.

        Linear weights N(0, 0.02), biases N(0, 0.01) (the reference zero-inits
        biases and the head, models.py:2259-2281, which would make any block math
        indistinguishable at the output), norm weights 1 + N(0, 0.1),
        modulations N(0, 1)/sqrt(dim).
        """
        import zlib
        shapes = SRDiT.param_shapes(cfg)

        def make(name, shape):
            gen = torch.Generator(device=device)
            gen.manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
            if name.endswith("modulation"):
                return torch.randn(shape, generator=gen, device=device) / cfg.dim ** 0.5
            if "norm" in name:
                t = 1 + 0.1 * torch.randn(shape, generator=gen, device=device)
            elif name.endswith("bias"):
                t = torch.randn(shape, generator=gen, device=device) * 0.01
            else:
                t = torch.randn(shape, generator=gen, device=device) * 0.02
            return t.to(torch.bfloat16)

        class LazySD(dict):
            def __missing__(self, key):
                return make(key, shapes[key])

        return LazySD()

    @classmethod
    def random_init(cls, cfg: SRDiTConfig, device="cuda", seed=0, **kw):
        """The model with ``seeded_state_dict`` weights."""
        return cls(cfg, SRDiT.seeded_state_dict(cfg, device, seed), device, **kw)

    @classmethod
    def from_state_dict(cls, cfg: SRDiTConfig, sd: dict, device="cuda"):
        return cls(cfg, sd, device)

    # ------------------------------------------------------------------ helpers
    def _make_layer(self, sd, prefix):
        return _Layer(sd, prefix, self.cfg, self.device)

    def _buf(self, name, shape, dtype):
        t = self._bufs.get(name)
        if t is None or t.shape != torch.Size(shape) or t.dtype != dtype:
            t = self._bufs[name] = torch.empty(shape, dtype=dtype, device=self.device)
        return t

    def new_cache(self, frame_tokens, grid_hw=None):
        """K/V ring for this model's heads (all heads; a tensor-parallel rank's slice)
        for frames of ``frame_tokens`` tokens (``grid_hw``: their (h, w) token grid,
        which a spatially partitioned model needs)."""
        c = self.cfg
        return KVRing(c.num_layers, frame_tokens, self.kv_width, c.kv_len, c.chunk_frames,
                      self.device)

    @property
    def kv_width(self):
        return self.cfg.dim

    def _cross_plan(self, M, Lc):
        """Dense cross attention as one 'window' per query row of a (1, M/W, W) grid
        against a (1, Lc/Wk, Wk) text grid."""
        key = (M, Lc)
        if key not in self._cross_plans:
            wq = max(d for d in range(8, 129, 8) if M % d == 0) if M % 8 == 0 else None
            wk = max(d for d in range(8, 129, 8) if Lc % d == 0) if Lc % 8 == 0 else None
            if wq is None or wk is None:
                raise _lib.SrditError(f"cross attention needs token counts divisible by 8 "
                                      f"(got {M}, {Lc})")
            hq, hk = M // wq, Lc // wk
            rows = [[0, 1, i, 0, 1, wq, 0, 1, 0, hk, 0, wk, 0, 0, 0, 0, 0, 1, 1] for i in range(hq)]
            params = torch.tensor(rows, dtype=torch.int32)
            tiling = ops.winattn_plan(params, blockgrid.P_PLAIN, 0)
            self._cross_plans[key] = (params.to(self.device), tiling, hq, wq, hk, wk)
        return self._cross_plans[key]

    def embed(self, latent, t, context, ctx_emb=None):
        """Patch, time and text embeddings (models.py:1827-1875) for one sample.

        latent [C, F, H, W] bf16; t scalar timestep; context [Lc, text_dim] bf16
        (or ``ctx_emb``, its text embedding computed earlier).
        Returns x [F*h*w, D] bf16, e0 [6, D] fp32, e [D] fp32, ctx [Lc, D] bf16, (f, h, w).
        """
        c = self.cfg
        x = torch.nn.functional.conv3d(latent[None].to(torch.bfloat16), self.patch_w,
                                       self.patch_b, stride=c.patch_size)
        f, h, w = x.shape[2:]
        x = x.flatten(2).transpose(1, 2)[0].contiguous()
        e0, e = self._time_embedding(t)
        if ctx_emb is not None:
            return x, e0, e, ctx_emb, (int(f), int(h), int(w))
        return x, e0, e, self.text_embedding(context), (int(f), int(h), int(w))

    def text_embedding(self, context):
        """text_embedding (Linear -> GELU(tanh) -> Linear) of the padded context."""
        c = self.cfg
        ctx = context.to(self.device, torch.bfloat16)
        if ctx.shape[0] < c.text_len:
            ctx = torch.cat([ctx, ctx.new_zeros(c.text_len - ctx.shape[0], ctx.shape[1])])
        ctx = torch.nn.functional.linear(ctx, *self.txt[0])
        ctx = torch.nn.functional.gelu(ctx, approximate="tanh")
        return torch.nn.functional.linear(ctx, *self.txt[1]).contiguous()

    def _time_embedding(self, t):
        """(e0 [6, D], e [D]) fp32 for timestep t, computed once per t value (the
        refiner uses two: denoise and refresh), so a forward issues no host-to-
        device copy and can be captured in a CUDA graph."""
        key = float(t)
        hit = self._temb.get(key)
        if hit is None:
            c = self.cfg
            tt = torch.as_tensor([key], device=self.device)
            e = sinusoidal_embedding_1d(c.freq_dim, tt).float()
            e = torch.nn.functional.linear(e, *self.tim[0])
            e = torch.nn.functional.linear(torch.nn.functional.silu(e), *self.tim[1])
            e0 = torch.nn.functional.linear(torch.nn.functional.silu(e), *self.tproj)
            hit = self._temb[key] = (e0.view(6, c.dim).contiguous(), e[0].contiguous())
        return hit

    def set_t_offset(self, t_offset):
        """The temporal RoPE position of the chunk's first frame, in device memory
        (read by the kernels when they run)."""
        if t_offset < 0 or t_offset + self.cfg.chunk_frames > self.cfg.rope_rows:
            raise _lib.SrditError(f"temporal position {t_offset} outside the RoPE table")
        self.t_offset_dev.fill_(int(t_offset))

    def head(self, x, e, grid):
        """Head (models.py:1357-1384, fp32 as under autocast) + unpatchify (:2234-2257)."""
        c = self.cfg
        f, h, w = grid
        mod = self.head_mod + e[None]
        n = torch.nn.functional.layer_norm(x.float(), (c.dim,), eps=c.eps).to(torch.bfloat16)
        y = torch.nn.functional.linear(n.float() * (1 + mod[1]) + mod[0], self.head_w, self.head_b)
        p = c.patch_size
        y = y.view(f, h, w, *p, c.out_dim)
        y = torch.einsum("fhwpqrc->cfphqwr", y).reshape(c.out_dim, f * p[0], h * p[1], w * p[2])
        return y.to(torch.bfloat16)

    def _window_plan(self, f, f_kv, h, w, streaming, mode, independent_frames):
        """The window plan dict of a chunk of f frames on an h x w token grid over
        f_kv visible frames (``independent_frames``: f separate 1-frame samples)."""
        from .attention import cached_plan, frames_plan
        c = self.cfg
        if independent_frames:
            spec1 = blockgrid.make_spec(f_cur=1, f_kv=1, h=h, w=w, block_t=c.block_t,
                                        block_hw=c.block_hw, block_radius_hw=c.block_radius_hw,
                                        block_radius_t=c.block_radius_t, streaming=False)
            return frames_plan(spec1, f)
        spec = blockgrid.make_spec(f_cur=f, f_kv=f_kv, h=h, w=w, block_t=c.block_t,
                                   block_hw=c.block_hw, block_radius_hw=c.block_radius_hw,
                                   block_radius_t=c.block_radius_t, streaming=streaming)
        return cached_plan(spec, mode)

    def _kv_width(self, w):
        """Token columns of the K/V ring's (and the anchor's) frames for a chunk w
        tokens wide: the chunk's own."""
        return w

    def _begin_forward(self):
        """Called at the start of every forward (a sharded model's per-forward setup)."""

    def _ring_kw(self, li, cache, w):
        """Extra ``rms_rope`` arguments of the K/V ring write of block ``li``."""
        return {}

    def _kv_sync(self, li, cache, slot_cur, f):
        """Called between block ``li``'s K/V ring write and its attention."""

    def _setup(self, latent, t, context, cache, anchor_kv, anchor_align, ctx_emb, n_heads,
               width, independent_frames=False):
        """Embeddings, the window plan and the attention geometries of one forward.

        ``n_heads`` / ``width``: the heads and row width of the q/k/v/out
        tensors this process holds (all heads, or a tensor-parallel slice)."""
        from types import SimpleNamespace
        c = self.cfg
        x, e0, e, ctx, grid = self.embed(latent, t, context, ctx_emb)
        f, h, w = grid
        L = h * w
        M = f * L
        dev = self.device
        if cache is None:
            cache = self._scratch_cache(L, (h, w))
            cache.reset()
        f_kv = cache.frames + f
        if f_kv > cache.cap:
            raise _lib.SrditError(f"chunk of {f} frames does not fit the ring of {cache.cap}")
        slot_cur = (cache.start + cache.frames) % cache.cap
        mode = None if anchor_kv is None else anchor_align
        from .attention import _plan_device_state
        if independent_frames and (cache.frames or anchor_kv is not None):
            raise _lib.SrditError("independent_frames: no cache and no anchor")
        plan = self._window_plan(f, f_kv, h, w, cache.frames > 0 or anchor_kv is not None, mode,
                                 independent_frames)
        kv_w = self._kv_width(w)
        fkey = ("flops", n_heads)
        if fkey not in plan:
            plan[fkey] = blockgrid.visible_flops(plan["params"], int(plan["p_stride"]),
                                                 n_heads, 128)
        a_hw = (h, kv_w) if anchor_kv is not None else None
        params_dev, tiling, n_w, amode, split_dev = _plan_device_state(
            plan, dev, mode, (f, h, w, f_kv, a_hw, f if a_hw else 0, kv_w),
            dict(f_cur=f, h=h, w=w, kv_frames=f_kv, a_hw=a_hw, a_frames=f if a_hw else 0,
                 kv_w=kv_w))
        geom = _lib.WinattnGeom()
        geom.q_frames, geom.q_h, geom.q_w = f, h, w
        geom.kv_h, geom.kv_w, geom.kv_slots, geom.kv_slot0 = h, kv_w, cache.cap, cache.start
        geom.n_heads, geom.head_dim = n_heads, 128
        geom.q_stride = geom.kv_stride = geom.o_stride = width
        geom.scale = 128 ** -0.5
        geom.col_split = None if split_dev is None else split_dev.data_ptr()
        if anchor_kv is not None:
            geom.a_frames, geom.a_h, geom.a_w, geom.a_stride = f, h, kv_w, width

        Lc = ctx.shape[0]
        cp_params, cp_tiling, cp_nw, cwq, chk, cwk = self._cross_plan(M, Lc)
        cgeom = _lib.WinattnGeom()
        cgeom.q_frames, cgeom.q_h, cgeom.q_w = 1, M // cwq, cwq
        cgeom.kv_h, cgeom.kv_w, cgeom.kv_slots, cgeom.kv_slot0 = chk, cwk, 1, 0
        cgeom.n_heads, cgeom.head_dim = n_heads, 128
        cgeom.q_stride = cgeom.o_stride = width
        cgeom.kv_stride = 2 * width
        cgeom.scale = 128 ** -0.5
        return SimpleNamespace(x=x, e0=e0, e=e, ctx=ctx, grid=grid, cache=cache, L=L, M=M,
                               Lc=Lc, slot_cur=slot_cur, plan=plan, params_dev=params_dev,
                               tiling=tiling, n_w=n_w, amode=amode, geom=geom,
                               cp_params=cp_params, cp_tiling=cp_tiling, cp_nw=cp_nw,
                               cgeom=cgeom, flops=plan[fkey],
                               cross_flops=4 * 128 * n_heads * M * Lc)

    # ------------------------------------------------------------------ forward
    def forward_chunk(self, latent, t, context, *, cache: KVRing | None = None,
                      t_offset=0, update_cache=False, anchor_kv=None, anchor_align="frame",
                      return_kv=False, ctx_emb=None, text: TextCache | None = None,
                      kv_only=False, independent_frames=False, block_outputs=None):
        """One streaming forward over a chunk (``_forward_inference`` for one sample).

        latent [C_in, f, H, W]; ``cache`` holds the previous chunks' K/V (read in
        place); ``update_cache=True`` makes this the cache-refresh forward (the
        chunk's K/V are kept, the ring advances). ``anchor_kv``: per-layer (K, V)
        [f*h*w, D] bf16 LQ anchor (never cached). ``return_kv`` returns the
        per-layer roped K / V of this chunk (the anchor harvest). ``text``: the
        context's ``text_cache`` (else the text embedding and cross K/V are
        computed here, as the reference does every forward). ``kv_only=True``
        (a cache-refresh forward whose prediction is discarded, as the refiner's
        t=0 pass is): the last block stops once its K/V are in the ring, only its
        k / v columns are projected, and nothing is returned -- the ring ends up
        exactly as after the full forward. ``independent_frames=True`` (no cache,
        no anchor): the chunk's frames are independent 1-frame samples -- frame j
        attends to frame j only, at temporal position t_offset + j -- which is the
        anchor harvest's batch (causal_inference.py:456-460) as one forward.
        ``block_outputs`` (a list, optional): every block's output hidden state
        [M, D] bf16 is appended to it (a copy; for parity checks per block).
        Returns the refined prediction [C_out, f, H, W] bf16 (and the K/V list).
        """
        if kv_only and (return_kv or not update_cache):
            raise _lib.SrditError("kv_only is for a cache-refresh forward (update_cache=True, "
                                  "no return_kv)")
        c = self.cfg
        ops = self.ops
        if not self.graph_capture:
            self.set_t_offset(t_offset)
        if text is not None:
            ctx_emb = text.ctx_emb
        S = self._setup(latent, t, context, cache, anchor_kv, anchor_align, ctx_emb,
                        c.num_heads, c.dim, independent_frames)
        self._begin_forward()
        x, e0, e, ctx, grid, cache = S.x, S.e0, S.e, S.ctx, S.grid, S.cache
        f, h, w = grid
        L, M, D, Lc = S.L, S.M, c.dim, S.Lc
        dev = self.device
        slot_cur, plan, params_dev, tiling, n_w, amode, geom = (
            S.slot_cur, S.plan, S.params_dev, S.tiling, S.n_w, S.amode, S.geom)
        cp_params, cp_tiling, cp_nw, cgeom = S.cp_params, S.cp_tiling, S.cp_nw, S.cgeom

        bf16, f32, f8 = torch.bfloat16, torch.float32, torch.float8_e4m3fn
        xq = self._buf("xq", (M, D), f8)
        xs = self._buf("xs", (M,), f32)
        qkv = self._buf("qkv", (M, 3 * D), bf16)
        qb = self._buf("q", (M, D), bf16)
        att = self._buf("att", (M, D), bf16)
        hbuf = self._buf("h", (M, c.ffn_dim), bf16)
        hq = self._buf("hq", (M, c.ffn_dim), f8)
        hs = self._buf("hs", (M,), f32)
        amax = self._buf("amax", (M,), f32)
        ckv = self._buf("ckv", (Lc, 2 * D), bf16)
        ctxq, ctxs = ops.quant_rowwise(ctx) if text is None else (None, None)
        mods = torch.stack([ly.modulation for ly in self.layers]) + e0[None]   # [layers, 6, D]
        # the GEMM can store V into ring slots (whole 32-row boxes of frames the
        # chunk's own size)
        v_direct = L % 32 == 0 and D % 64 == 0 and cache.frame_tokens == L
        kv_out = [] if return_kv else None
        st = self.status
        cos, sin = self.rope_cos, self.rope_sin
        for li, ly in enumerate(self.layers):
            em = mods[li]
            kr, vr = cache.k[li], cache.v[li]
            # --- self attention
            ops.ln_mod_quant(x, c.eps, shift=em[0], scale=em[1], q=xq, qscale=xs)
            # q | k | v projection; V goes straight into its ring slot (whole 32-row
            # store boxes per frame), else the K kernel copies it there
            last_kv = kv_only and li == len(self.layers) - 1
            c0 = D if last_kv else 0   # the refresh pass's last block: k | v only
            v_ring = (vr, 2 * D - c0, L, slot_cur, cache.cap) if v_direct else None
            ops.fp8_gemm(xq, xs, ly.w_qkv[c0:], ly.s_qkv[c0:], ly.b_qkv[c0:], qkv[:, c0:],
                         v_ring=v_ring)
            vcopy = {} if v_direct else dict(v_src=qkv[:, 2 * D:], v_dst=vr)
            ops.rms_rope(qkv[:, D:2 * D], ly.nk, c.eps, kr, frame_tokens=L, slot0=slot_cur,
                         n_slots=cache.cap, cos=cos, sin=sin, grid_h=h, grid_w=w,
                         t_offset_dev=self.t_offset_dev, w_offset=self.rope_w0, **vcopy,
                         **self._ring_kw(li, cache, w))
            if last_kv:
                self._kv_sync(li, cache, slot_cur, f)
                break   # its K / V are in the ring: nothing else of the block is used
            ops.rms_rope(qkv[:, :D], ly.nq, c.eps, qb, frame_tokens=L, cos=cos, sin=sin,
                         grid_h=h, grid_w=w, t_offset_dev=self.t_offset_dev,
                         w_offset=self.rope_w0)
            self._kv_sync(li, cache, slot_cur, f)
            ak = av = None
            if anchor_kv is not None:
                ak, av = anchor_kv[li]
            ops.winattn(qb, kr, vr, att, params_dev=params_dev, n_w=n_w,
                        p_stride=int(plan["p_stride"]), anchor_mode=amode, geom=geom,
                        tiling=tiling, k_anchor=ak, v_anchor=av, status=st,
                        flops=S.flops)
            if return_kv:
                idx = (torch.arange(f, device=dev) + slot_cur) % cache.cap
                Lr = cache.frame_tokens
                kv_out.append((kr.view(cache.cap, Lr, D)[idx].reshape(f * Lr, D).clone(),
                               vr.view(cache.cap, Lr, D)[idx].reshape(f * Lr, D).clone()))
            ops.quant_rowwise(att, q=xq, scale=xs)
            ops.fp8_gemm(xq, xs, ly.w_o, ly.s_o, ly.b_o, x, epilogue="gated_res", residual=x,
                         gate=em[2])
            # --- cross attention
            ops.ln_mod_quant(x, c.eps, ln_weight=ly.n3w, ln_bias=ly.n3b, q=xq, qscale=xs)
            ops.fp8_gemm(xq, xs, ly.w_cq, ly.s_cq, ly.b_cq, qb)
            ops.rms_rope(qb, ly.cnq, c.eps, qb, frame_tokens=M)
            if text is None:
                ops.fp8_gemm(ctxq, ctxs, ly.w_ckv, ly.s_ckv, ly.b_ckv, ckv)
                ops.rms_rope(ckv[:, :D], ly.cnk, c.eps, ckv[:, :D], frame_tokens=Lc)
            else:
                ckv = text.kv[li]
            ops.winattn(qb, ckv[:, :D], ckv[:, D:], att, params_dev=cp_params, n_w=cp_nw,
                        p_stride=blockgrid.P_PLAIN, anchor_mode=0, geom=cgeom, tiling=cp_tiling,
                        status=st, flops=S.cross_flops)
            ops.quant_rowwise(att, q=xq, scale=xs)
            ops.fp8_gemm(xq, xs, ly.w_co, ly.s_co, ly.b_co, x, epilogue="res", residual=x)
            # --- FFN
            ops.ln_mod_quant(x, c.eps, shift=em[3], scale=em[4], q=xq, qscale=xs)
            amax.zero_()
            ops.fp8_gemm(xq, xs, ly.w_f0, ly.s_f0, ly.b_f0, hbuf, epilogue="gelu", row_amax=amax)
            ops.quant_rowwise(hbuf, amax=amax, q=hq, scale=hs)
            ops.fp8_gemm(hq, hs, ly.w_f2, ly.s_f2, ly.b_f2, x, epilogue="gated_res", residual=x,
                         gate=em[5])
            if block_outputs is not None:
                block_outputs.append(x.clone())
        if update_cache:
            cache.commit(f)
        if kv_only:
            return None
        out = self.head(x, e, grid)
        return (out, kv_out) if return_kv else out

    # ------------------------------------------------------------------ text cache
    def text_cache(self, context, into=None):
        """The context's text embedding and every block's cross-attention K | V
        (cross_attn.k / .v, norm_k on K), computed once per context.

        The refiner's text context is fixed for a clip, yet the reference
        recomputes these in every forward (models.py:1048-1054, :1854-1866); the
        values are the same, so a forward given the cache skips that work.
        ``into``: a previous cache to overwrite in place (its buffers stay put,
        which keeps captured CUDA graphs valid). Returns the cache."""
        ops = self.ops
        c = self.cfg
        ctx = self.text_embedding(context)
        Lc, W = ctx.shape[0], self.kv_width
        if into is None:
            into = TextCache(ctx.clone(), [torch.empty(Lc, 2 * W, dtype=torch.bfloat16,
                                                       device=self.device)
                                           for _ in self.layers])
        else:
            into.ctx_emb.copy_(ctx)
        ctxq, ctxs = ops.quant_rowwise(into.ctx_emb)
        for li, ly in enumerate(self.layers):
            self._text_kv(ly, ctxq, ctxs, into.kv[li])
        return into

    def _text_kv(self, ly, ctxq, ctxs, ckv):
        c = self.cfg
        W = self.kv_width
        self.ops.fp8_gemm(ctxq, ctxs, ly.w_ckv, ly.s_ckv, ly.b_ckv, ckv)
        self.ops.rms_rope(ckv[:, :W], ly.cnk, c.eps, ckv[:, :W], frame_tokens=ckv.shape[0])

    def _scratch_cache(self, L, grid_hw=None):
        key = ("scratch_cache", L)
        if key not in self._bufs:
            self._bufs[key] = self.new_cache(L)
        return self._bufs[key]

    def check_status(self):
        """Raise if a kernel reported a bounded wait that ran out."""
        v = int(self.status.item())
        if v:
            self.status.zero_()
            raise _lib.SrditError(f"a kernel gave up on a device-side wait (status {v})")
