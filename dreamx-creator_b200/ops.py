"""Tensor-level wrappers over the C ABI (torch tensors in, device pointers out).

Each function validates dtype / device / layout, then calls exactly one entry
point of libsrdit_b200.so on the current CUDA stream. Nothing here computes:
there is no fallback when the library or a GPU is missing.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

EPILOGUES = {"store": _lib.SRDIT_EPI_STORE, "gelu": _lib.SRDIT_EPI_GELU,
             "gated_res": _lib.SRDIT_EPI_GATED_RES, "res": _lib.SRDIT_EPI_RES}


class Stats:
    """Launch accounting.

    ``launches`` counts the kernels this module launched. When ``events`` is a
    list, every launch appends ``(kind, start_event, end_event, work)``, the
    events recorded on the launching stream around the launch and ``work`` its
    algorithmic FLOPs (GEMM, attention) or bytes (row kernels), so a profiling
    pass can attribute time per kernel kind. Leave it None in timed regions:
    the event records themselves cost time.
    """
    launches = 0
    events = None


def _launch(name, *args, kind=None, work=0):
    ev = Stats.events
    if ev is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
    _lib.call(name, *args)
    Stats.launches += 1
    if ev is not None:
        e1.record()
        ev.append((kind or name, e0, e1, int(work)))


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise _lib.SrditError("the B200 kernels need CUDA tensors (there is no CPU path)")


def _rows(t: torch.Tensor):
    """(row stride in elements) of a 2-D row-major view with unit inner stride."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise _lib.SrditError(f"expected a 2-D row-major tensor, got shape {tuple(t.shape)} "
                              f"strides {t.stride()}")
    return t.stride(0)


def fp8_gemm(a_fp8, a_scale, w_fp8, w_scale, bias=None, out=None, *, epilogue="store",
             residual=None, gate=None, row_amax=None, status=None, v_ring=None):
    """out[M,N] = epilogue(a_fp8 @ w_fp8^T * a_scale[:,None] * w_scale[None,:] + bias).

    ``v_ring`` (STORE only): (ring [slots*frame_tokens, W] bf16, col0, frame_tokens,
    slot0, n_slots) -- columns [col0, N) go into the frame ring (output frame f
    into slot (slot0 + f) % n_slots) instead of ``out``."""
    _need_cuda(a_fp8, a_scale, w_fp8, w_scale, bias, out, residual, gate, row_amax)
    if a_fp8.dtype != torch.float8_e4m3fn or w_fp8.dtype != torch.float8_e4m3fn:
        raise _lib.SrditError("fp8_gemm operands must be float8_e4m3fn")
    M, K = a_fp8.shape
    N, K2 = w_fp8.shape
    if K != K2:
        raise _lib.SrditError(f"K mismatch {K} vs {K2}")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a_fp8.device)
    for t, nm in ((a_scale, "a_scale"), (w_scale, "w_scale"), (gate, "gate"),
                  (row_amax, "row_amax")):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
            raise _lib.SrditError(f"{nm} must be contiguous float32")
    if bias is not None and (bias.dtype != torch.bfloat16 or not bias.is_contiguous()):
        raise _lib.SrditError("bias must be contiguous bf16")
    if v_ring is not None:
        if epilogue != "store":
            raise _lib.SrditError("v_ring needs the store epilogue")
        ring, col0, frame_tokens, slot0, n_slots = v_ring
        _need_cuda(ring)
        if ring.dtype != torch.bfloat16:
            raise _lib.SrditError("the V ring is bf16")
        vr = _lib.VRing(ctypes.c_void_p(ring.data_ptr()), _rows(ring), int(col0),
                        int(frame_tokens), int(slot0), int(n_slots))
        _launch("srdit_fp8_gemm_vring", _ptr(a_fp8), _ptr(a_scale), _ptr(w_fp8), _ptr(w_scale),
                _ptr(bias), _ptr(out), M, N, K, _rows(a_fp8), _rows(w_fp8), _rows(out),
                ctypes.byref(vr), _ptr(status), _stream(a_fp8.device), kind="fp8_gemm",
                work=2 * M * N * K)
        return out
    ldr = _rows(residual) if residual is not None else 0
    _launch("srdit_fp8_gemm", _ptr(a_fp8), _ptr(a_scale), _ptr(w_fp8), _ptr(w_scale),
            _ptr(bias), _ptr(out), M, N, K, _rows(a_fp8), _rows(w_fp8), _rows(out),
            EPILOGUES[epilogue], _ptr(residual), ldr, _ptr(gate), _ptr(row_amax),
            _ptr(status), _stream(a_fp8.device), kind="fp8_gemm", work=2 * M * N * K)
    return out


def quant_rowwise(x, amax=None, q=None, scale=None):
    """(e4m3 [M,K], fp32 scale [M]) of a bf16 [M,K] matrix (fp8_linear.py:93-103)."""
    _need_cuda(x, amax, q, scale)
    if x.dtype != torch.bfloat16:
        raise _lib.SrditError("quant_rowwise takes bf16")
    M, K = x.shape
    if q is None:
        q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty(M, dtype=torch.float32, device=x.device)
    _launch("srdit_quant_rowwise", _ptr(x), _rows(x), M, K, _ptr(amax), _ptr(q), _rows(q),
            _ptr(scale), _stream(x.device), kind="quant_rowwise",
            work=M * K * 3 + 4 * M)
    return q, scale


def ln_mod_quant(x, eps=1e-6, *, ln_weight=None, ln_bias=None, shift=None, scale=None,
                 q=None, qscale=None):
    """LayerNorm (+affine) -> bf16 -> adaLN modulate -> row-wise e4m3."""
    _need_cuda(x, ln_weight, ln_bias, shift, scale, q, qscale)
    if x.dtype != torch.bfloat16:
        raise _lib.SrditError("ln_mod_quant takes bf16")
    M, K = x.shape
    if q is None:
        q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    if qscale is None:
        qscale = torch.empty(M, dtype=torch.float32, device=x.device)
    _launch("srdit_ln_mod_quant", _ptr(x), _rows(x), M, K, float(eps), _ptr(ln_weight),
            _ptr(ln_bias), _ptr(shift), _ptr(scale), _ptr(q), _rows(q), _ptr(qscale),
            _stream(x.device), kind="ln_mod_quant", work=M * K * 2 + M * K + 4 * M)
    return q, qscale


def rms_rope(src, weight, eps, dst, *, frame_tokens, slot0=0, n_slots=1 << 30, cos=None,
             sin=None, grid_h=0, grid_w=0, t_offset=0, v_src=None, v_dst=None, ss=None,
             norm_width=0, t_offset_dev=None, w_offset=0, dst_grid_w=0, dst_w0=0, halo=None):
    """RMSNorm(src) * weight [-> 3-D RoPE] -> dst frame slots (+ V copy).

    ``ss`` ([M] fp32, optional): per-row sum of squares over ``norm_width``
    columns (a tensor-parallel slice's all-reduced statistic). ``t_offset_dev``
    (optional int32 [1] on the device): added to ``t_offset`` at run time.
    ``w_offset``: width position of the grid's column 0 (a strip of a wider grid).
    ``dst_grid_w`` > 0: destination frames of grid_h x dst_grid_w tokens, the
    grid's column c written to column c + ``dst_w0``. ``halo`` (a ``_lib.RopeHalo``):
    the strip's edge columns also stored into the neighbours' rings, then signalled."""
    _need_cuda(src, weight, dst, cos, sin, v_src, v_dst, ss)
    if ss is not None and (ss.dtype != torch.float32 or not ss.is_contiguous()):
        raise _lib.SrditError("ss must be contiguous float32")
    M, K = src.shape
    if cos is not None and (cos.dtype != torch.float64 or sin.dtype != torch.float64
                            or cos.shape != sin.shape or cos.shape[1] != 64
                            or not cos.is_contiguous() or not sin.is_contiguous()):
        raise _lib.SrditError("RoPE tables must be contiguous float64 [rows, 64]")
    tab_rows = cos.shape[0] if cos is not None else 0
    _launch("srdit_rms_rope", _ptr(src), _rows(src), M, K, _ptr(weight), float(eps),
            _ptr(dst), _rows(dst), int(frame_tokens), int(slot0), int(n_slots), _ptr(cos),
            _ptr(sin), int(tab_rows), int(grid_h), int(grid_w), int(t_offset), _ptr(v_src),
            _rows(v_src) if v_src is not None else 0, _ptr(v_dst),
            _rows(v_dst) if v_dst is not None else 0, _ptr(ss), int(norm_width),
            _ptr(t_offset_dev), int(w_offset), int(dst_grid_w), int(dst_w0),
            ctypes.byref(halo) if halo is not None else None,
            _stream(src.device), kind="rms_rope",
            work=M * K * 2 * (4 if v_src is not None else 2))
    return dst


def row_reduce(x, op, out=None):
    """Per-row sum of squares (op "sumsq") or max |x| (op "absmax") of a bf16 [M, K]."""
    _need_cuda(x, out)
    if x.dtype != torch.bfloat16:
        raise _lib.SrditError("row_reduce takes bf16")
    M, K = x.shape
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    code = {"sumsq": _lib.SRDIT_ROW_SUMSQ, "absmax": _lib.SRDIT_ROW_ABSMAX}[op]
    _launch("srdit_row_reduce", _ptr(x), _rows(x), M, K, code, _ptr(out), _stream(x.device),
            kind="row_reduce", work=M * K * 2 + 4 * M)
    return out


def residual(x, parts, bias=None, gate=None):
    """x = bf16(x + bf16(sum(parts) + bias) [* gate]) in place; parts [S, M, N] or [M, N]."""
    _need_cuda(x, parts, bias, gate)
    p3 = parts if parts.dim() == 3 else parts.unsqueeze(0)
    if p3.dtype != torch.bfloat16 or p3.stride(2) != 1:
        raise _lib.SrditError("residual parts must be bf16 with unit inner stride")
    S, M, N = p3.shape
    if x.shape != (M, N):
        raise _lib.SrditError(f"x {tuple(x.shape)} vs parts {tuple(p3.shape)}")
    if gate is not None and (gate.dtype != torch.float32 or not gate.is_contiguous()):
        raise _lib.SrditError("gate must be contiguous float32")
    _launch("srdit_residual", _ptr(x), _rows(x), M, N, _ptr(p3), S, p3.stride(0), p3.stride(1),
            _ptr(bias), _ptr(gate), _stream(x.device), kind="residual",
            work=M * N * 2 * (S + 2))
    return x


def winattn_plan(params_host: torch.Tensor, p_stride: int, anchor_mode: int):
    """Tiling of a window plan (int32 [n_w, p_stride] rows on the host)."""
    p = params_host.contiguous()
    if p.dtype != torch.int32 or p.device.type != "cpu":
        raise _lib.SrditError("params rows must be a CPU int32 tensor")
    t = _lib.WinattnTiling()
    _lib.call("srdit_winattn_plan", ctypes.c_void_p(p.data_ptr()), p.shape[0], int(p_stride),
              int(anchor_mode), ctypes.byref(t))
    return t


def winattn(q, k_hr, v_hr, out, *, params_dev, n_w, p_stride, anchor_mode, geom, tiling,
            k_anchor=None, v_anchor=None, status=None, flops=0):
    """One window-attention launch (see include/srdit_b200.h, srdit_winattn_fwd).
    ``flops``: the launch's visible-pair FLOPs, for launch accounting only."""
    _need_cuda(q, k_hr, v_hr, out, params_dev, k_anchor, v_anchor)
    for t in (q, k_hr, v_hr, out, k_anchor, v_anchor):
        if t is not None and t.dtype != torch.bfloat16:
            raise _lib.SrditError("window attention takes bf16 q/k/v")
    _launch("srdit_winattn_fwd", _ptr(q), _ptr(k_hr), _ptr(v_hr), _ptr(k_anchor),
            _ptr(v_anchor), _ptr(out), _ptr(params_dev), int(n_w), int(p_stride),
            int(anchor_mode), ctypes.byref(geom), ctypes.byref(tiling), _ptr(status),
            _stream(q.device), kind="winattn", work=flops)
    return out


# --------------------------------------------------------------------------- tensor parallel
def peer_ptrs(ptrs):
    """ctypes table of per-rank device addresses (ints)."""
    t = _lib.PeerPtrs()
    for i, v in enumerate(ptrs):
        t.p[i] = int(v)
    return t


def fp8_gemm_ctas(M, N):
    return _lib.count("srdit_fp8_gemm_ctas", int(M), int(N))


def fp8_gemm_tp(a_fp8, a_scale, w_fp8, w_scale, bias=None, out=None, *, tp, epilogue="store",
                row_amax=None, status=None):
    """srdit_fp8_gemm_tp: ``tp`` is a filled ``_lib.TpGemm``; epilogue "peer" stores the
    partial into the owners' receive slots (``out`` unused)."""
    _need_cuda(a_fp8, a_scale, w_fp8, w_scale, bias, out, row_amax)
    M, K = a_fp8.shape
    N = w_fp8.shape[0]
    code = {"store": _lib.SRDIT_EPI_STORE, "gelu": _lib.SRDIT_EPI_GELU,
            "peer": _lib.SRDIT_EPI_PEER}[epilogue]
    ldo = _rows(out) if out is not None else 0
    _launch("srdit_fp8_gemm_tp", _ptr(a_fp8), _ptr(a_scale), _ptr(w_fp8), _ptr(w_scale),
            _ptr(bias), _ptr(out), M, N, K, _rows(a_fp8), _rows(w_fp8), ldo, code,
            _ptr(row_amax), ctypes.byref(tp), _ptr(status), _stream(a_fp8.device),
            kind="fp8_gemm", work=2 * M * N * K)
    return out


def residual_tp(x, parts, *, bias=None, gate=None, flags, expected, status=None):
    """srdit_residual_tp over the receive buffer ``parts`` [S, M, N]."""
    _need_cuda(x, parts, bias, gate)
    S, M, N = parts.shape
    _launch("srdit_residual_tp", _ptr(x), _rows(x), M, N, _ptr(parts), S, parts.stride(0),
            parts.stride(1), _ptr(bias), _ptr(gate), ctypes.c_void_p(int(flags)),
            int(expected) & 0xffffffff, _ptr(status), _stream(x.device), kind="residual",
            work=M * N * 2 * (S + 2))
    return x


def tp_allreduce(t, op, *, slots, flags, rank, world, epoch, status=None):
    """In-place all-reduce (op "sum" / "max") of a contiguous fp32 vector through peer memory."""
    _need_cuda(t)
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise _lib.SrditError("tp_allreduce takes a contiguous float32 vector")
    code = {"sum": _lib.SRDIT_RED_SUM, "max": _lib.SRDIT_RED_MAX}[op]
    _launch("srdit_tp_allreduce", _ptr(t), _ptr(t), t.numel(), code, ctypes.byref(slots),
            ctypes.byref(flags), int(rank), int(world), int(epoch) & 0xffffffff, _ptr(status),
            _stream(t.device), kind="allreduce", work=t.numel() * 4 * world)
    return t


def conv3x3(x, weight, bias, *, frames_per_clip, n_src=1, replicate=True, residual=None,
            res_scale=1.0, relu=False, shuffle=1, out=None, status=None):
    """srdit_conv3x3 of channels-last frames x [F, H, W, cin] bf16 (cin a multiple of
    64) with ``weight`` [cout, n_src * 9 * cin] bf16 (``conv_weight`` builds it) and
    fp32 ``bias`` [cout]; returns out [F, H, W, cout], or [F, r H, r W, cout / r^2]
    with ``shuffle`` = r."""
    _need_cuda(x, weight, bias, residual, out, status)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or bias.dtype != torch.float32:
        raise _lib.SrditError("conv3x3 takes bf16 frames and weights and fp32 bias")
    if x.dim() != 4 or not x.is_contiguous() or not weight.is_contiguous():
        raise _lib.SrditError("conv3x3 takes contiguous [F, H, W, C] frames")
    F, H, W, cin = x.shape
    cout = weight.shape[0]
    if weight.shape[1] != n_src * 9 * cin or bias.shape != (cout,):
        raise _lib.SrditError(f"weight {tuple(weight.shape)} / bias {tuple(bias.shape)} do not "
                              f"match {n_src} source(s) of {cin} channels")
    r = int(shuffle)
    shape = (F, H, W, cout) if r == 1 else (F, r * H, r * W, cout // (r * r))
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
    elif tuple(out.shape) != shape or not out.is_contiguous() or out.dtype != torch.bfloat16:
        raise _lib.SrditError(f"out must be a contiguous bf16 {shape}")
    if residual is not None and (tuple(residual.shape) != (F, H, W, cout)
                                 or not residual.is_contiguous()
                                 or residual.dtype != torch.bfloat16):
        raise _lib.SrditError(f"residual must be a contiguous bf16 {(F, H, W, cout)}")
    _launch("srdit_conv3x3", _ptr(x), F, int(frames_per_clip), H, W, cin, int(n_src),
            int(bool(replicate)), _ptr(weight), _ptr(bias), cout, _ptr(residual),
            float(res_scale), int(bool(relu)), r, _ptr(out), _ptr(status), _stream(x.device),
            kind="conv3x3", work=2 * F * H * W * cout * n_src * 9 * cin)
    return out


def conv3d(x, weight, bias, *, kt=1, kh=3, residual=None, res_scale=1.0, relu=False,
           shuffle=1, shuffle_t=1, up2_phase=-1, dup=None, out=None, status=None):
    """srdit_conv3d: x [in_frames, H, W, cin] bf16 (the causal history of kt - 1
    frames first), ``weight`` [cout, kt * kh * kh * cin] bf16 (``conv3d_weight``),
    fp32 ``bias``; returns out [in_frames - kt + 1, H, W, cout] (shuffled shapes
    as the header states; with ``up2_phase`` >= 0 the caller passes ``out`` of
    the upsampled size, of which this launch writes one sub-pixel). ``dup`` =
    (block input [frames, H, W, cin], ft, shift): a phase launch's DupUp3D
    residual, gathered in the epilogue."""
    _need_cuda(x, weight, bias, residual, out, status)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or bias.dtype != torch.float32:
        raise _lib.SrditError("conv3d takes bf16 frames and weights and fp32 bias")
    if x.dim() != 4 or not x.is_contiguous() or not weight.is_contiguous():
        raise _lib.SrditError("conv3d takes contiguous [F, H, W, C] frames")
    Fi, H, W, cin = x.shape
    Fo = Fi - kt + 1
    cout = weight.shape[0]
    if weight.shape[1] != kt * kh * kh * cin or bias.shape != (cout,):
        raise _lib.SrditError(f"weight {tuple(weight.shape)} / bias {tuple(bias.shape)} do not "
                              f"match a {kt}x{kh}x{kh} conv of {cin} channels")
    r, st = int(shuffle), int(shuffle_t)
    if up2_phase >= 0:
        shape = (Fo, 2 * H, 2 * W, cout)
        if out is None:
            raise _lib.SrditError("an up2_phase launch writes into a given out")
    else:
        shape = (Fo * st, r * H, r * W, cout // (r * r * st))
    if out is None:
        out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
    elif tuple(out.shape) != shape or not out.is_contiguous() or out.dtype != torch.bfloat16:
        raise _lib.SrditError(f"out must be a contiguous bf16 {shape}")
    if residual is not None and (tuple(residual.shape) != tuple(out.shape)
                                 or not residual.is_contiguous()
                                 or residual.dtype != torch.bfloat16):
        raise _lib.SrditError(f"residual must be a contiguous bf16 {tuple(out.shape)}")
    a = _lib.Conv3dArgs()
    a.x, a.in_frames, a.out_frames, a.H, a.W, a.cin = x.data_ptr(), Fi, Fo, H, W, cin
    a.kt, a.kh, a.weight, a.bias, a.cout = kt, kh, weight.data_ptr(), bias.data_ptr(), cout
    a.residual = residual.data_ptr() if residual is not None else None
    a.res_scale, a.relu, a.shuffle, a.shuffle_t = float(res_scale), int(bool(relu)), r, st
    a.up2_phase, a.out = int(up2_phase), out.data_ptr()
    if dup is not None:
        xd, ft, shift = dup
        _need_cuda(xd)
        if (xd.dim() != 4 or tuple(xd.shape[1:3]) != (H, W) or not xd.is_contiguous()
                or xd.dtype != torch.bfloat16):
            raise _lib.SrditError(f"the DupUp3D source must be contiguous bf16 [frames, {H}, "
                                  f"{W}, cin], got {tuple(xd.shape)}")
        reps = cout * 4 * ft // xd.shape[3]
        du = _lib.DupUp(ctypes.c_void_p(xd.data_ptr()), xd.shape[0], xd.shape[3], int(ft),
                        int(reps), int(shift))
        a.dup = ctypes.pointer(du)
    a.status = status.data_ptr() if status is not None else None
    _launch("srdit_conv3d", ctypes.byref(a), _stream(x.device), kind="conv3d",
            work=2 * Fo * H * W * cout * kt * kh * kh * cin)
    return out


def conv3d_weight(w, *, cin_pad=None):
    """A Conv3d weight [cout, cin, kt, kh, kw] (or Conv2d [cout, cin, kh, kw]) as
    srdit_conv3d's K-major [cout, kt * kh * kw * cin_pad] bf16 matrix (column
    ((dt * kh + ky) * kw + kx) * cin_pad + c; channels past cin zero)."""
    if w.dim() == 4:
        w = w[:, :, None]
    cout, cin, kt, kh, kw = w.shape
    cin_pad = cin if cin_pad is None else int(cin_pad)
    t = w.detach().to(torch.float32).permute(0, 2, 3, 4, 1)
    if cin_pad != cin:
        t = torch.nn.functional.pad(t, (0, cin_pad - cin))
    return t.reshape(cout, kt * kh * kw * cin_pad).to(torch.bfloat16).contiguous()


def rms_silu(x, gamma, *, silu=True, out=None):
    """srdit_rms_silu over the channels of [..., C] bf16 frames (WanVAE RMS_norm, then
    SiLU); ``out`` may be x or a same-shaped view of another buffer."""
    _need_cuda(x, gamma, out)
    if (x.dtype != torch.bfloat16 or gamma.dtype != torch.bfloat16 or not x.is_contiguous()
            or not gamma.is_contiguous()):
        raise _lib.SrditError("rms_silu takes contiguous bf16 frames and a contiguous bf16 gamma")
    C = x.shape[-1]
    if gamma.numel() != C:
        raise _lib.SrditError(f"gamma of {gamma.numel()} for {C} channels")
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or not out.is_contiguous() or out.dtype != torch.bfloat16:
        raise _lib.SrditError("out must be a contiguous bf16 tensor of x's shape")
    P = x.numel() // C
    _launch("srdit_rms_silu", _ptr(x), P, C, _ptr(gamma), int(bool(silu)),
            _ptr(out), _stream(x.device), kind="rms_silu", work=4 * x.numel())
    return out


def conv_weight(w, *, n_src=1, cin_pad=None, shuffle=1):
    """An nn.Conv2d weight [cout, n_src * cin, 3, 3] as srdit_conv3x3's K-major
    [cout, n_src * 9 * cin_pad] bf16 matrix (column (s * 9 + ky * 3 + kx) * cin_pad
    + c; channels past cin zero). With ``shuffle`` = r the rows are reordered
    so that row g * cg + c holds output channel c * r^2 + g -- PixelShuffle(r)'s
    channel for sub-pixel g -- as the kernel's shuffled store expects."""
    cout, cin_all, kh, kw = w.shape
    if (kh, kw) != (3, 3) or cin_all % n_src:
        raise _lib.SrditError(f"not a 3x3 conv weight of {n_src} source(s): {tuple(w.shape)}")
    cin = cin_all // n_src
    cin_pad = cin if cin_pad is None else int(cin_pad)
    t = w.detach().to(torch.float32).reshape(cout, n_src, cin, 3, 3).permute(0, 1, 3, 4, 2)
    if cin_pad != cin:
        t = torch.nn.functional.pad(t, (0, cin_pad - cin))
    t = t.reshape(cout, n_src * 9 * cin_pad)
    r = int(shuffle)
    if r > 1:
        cg = cout // (r * r)
        t = t.reshape(cg, r * r, -1).transpose(0, 1).reshape(cout, -1)
    return t.to(torch.bfloat16).contiguous()


def conv_bias(b, *, shuffle=1):
    """The conv's bias [cout] as fp32, in ``conv_weight``'s row order."""
    t = b.detach().to(torch.float32)
    r = int(shuffle)
    if r > 1:
        t = t.reshape(-1, r * r).t().reshape(-1)
    return t.contiguous()


def wait_counters(counters: int, mask: int, expected: int, *, status=None, device=None):
    """srdit_wait_counters: the stream waits (bounded) until the uint32 counters at
    device address ``counters`` selected by ``mask`` reach ``expected``."""
    _need_cuda(status)
    _launch("srdit_wait_counters", ctypes.c_void_p(int(counters)), int(mask) & 0xffffffff,
            int(expected) & 0xffffffff, _ptr(status), _stream(device), kind="wait")


def ln_mod_quant_tp(x, eps=1e-6, *, ln_weight=None, ln_bias=None, shift=None, scale=None,
                    q_rows, s_rows, flags, done, rank, world, ldq):
    """srdit_ln_mod_quant_tp: this rank's LN-modulate-quant rows stored into every
    rank's gather buffer (``q_rows`` / ``s_rows`` peer tables), then ``flags``
    signalled; ``done`` is a zeroed uint32 tensor of this rank."""
    _need_cuda(x, ln_weight, ln_bias, shift, scale, done)
    if x.dtype != torch.bfloat16:
        raise _lib.SrditError("ln_mod_quant takes bf16")
    M, K = x.shape
    _launch("srdit_ln_mod_quant_tp", _ptr(x), _rows(x), M, K, float(eps), _ptr(ln_weight),
            _ptr(ln_bias), _ptr(shift), _ptr(scale), int(ldq), ctypes.byref(q_rows),
            ctypes.byref(s_rows), ctypes.byref(flags), _ptr(done), int(rank), int(world),
            _stream(x.device), kind="ln_mod_quant", work=M * K * 2 + (M * K + 4 * M) * world)


def tp_push(src, dst, src2, dst2, *, flags, rank, world, stream=None):
    """srdit_tp_push: copy-engine pushes of src (and src2) to every other rank's
    dst / dst2 addresses (``peer_ptrs`` tables), then signal ``flags``."""
    _need_cuda(src, src2)
    st = ctypes.c_void_p((stream or torch.cuda.current_stream(src.device)).cuda_stream)
    _lib.call("srdit_tp_push", _ptr(src), ctypes.byref(dst), src.numel() * src.element_size(),
              _ptr(src2), ctypes.byref(dst2) if dst2 is not None else None,
              (src2.numel() * src2.element_size()) if src2 is not None else 0,
              ctypes.byref(flags), int(rank), int(world), st)
    Stats.launches += 1


def ipc_handle(t):
    """(64-byte CUDA IPC handle, byte offset) of the allocation holding tensor ``t``."""
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_ulonglong(0)
    _lib.call("srdit_ipc_handle", _ptr(t), h, ctypes.byref(off))
    return bytes(h.raw), int(off.value)


def ipc_open(handle: bytes) -> int:
    """Map a peer's allocation; returns its base address in this process."""
    buf = ctypes.create_string_buffer(handle, 64)
    ptr = ctypes.c_void_p()
    _lib.call("srdit_ipc_open", buf, ctypes.byref(ptr))
    return int(ptr.value)


def ipc_close(addr: int) -> None:
    _lib.call("srdit_ipc_close", ctypes.c_void_p(addr))
