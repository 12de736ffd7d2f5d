"""ctypes binding of libsrdit_b200.so.

The library is the only compute path of this package: there is no CPU or
PyTorch fallback. ``lib()`` raises if the shared object is missing or does not
export every entry point of ``include/srdit_b200.h``; every call raises
``SrditError`` on a non-zero return code.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libsrdit_b200.so"
HEADER = PKG.parent / "include" / "srdit_b200.h"

SRDIT_EPI_STORE, SRDIT_EPI_GELU, SRDIT_EPI_GATED_RES, SRDIT_EPI_RES = 0, 1, 2, 3
SRDIT_P_FRAME, SRDIT_P_PLAIN = 17, 19
SRDIT_ANCHOR_NONE, SRDIT_ANCHOR_CHUNK, SRDIT_ANCHOR_FRAME = 0, 1, 2
SRDIT_STATUS_TIMEOUT = 1
SRDIT_SPLIT_FIELDS = 9
SRDIT_ROW_SUMSQ, SRDIT_ROW_ABSMAX = 0, 1

c_int, c_ll, c_float, c_vp = ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_void_p


class WinattnGeom(ctypes.Structure):
    _fields_ = [("q_frames", c_int), ("q_h", c_int), ("q_w", c_int),
                ("kv_h", c_int), ("kv_w", c_int), ("kv_slots", c_int), ("kv_slot0", c_int),
                ("a_frames", c_int), ("a_h", c_int), ("a_w", c_int),
                ("n_heads", c_int), ("head_dim", c_int),
                ("q_stride", c_ll), ("kv_stride", c_ll), ("a_stride", c_ll),
                ("o_stride", c_ll), ("scale", c_float), ("col_split", c_vp),
                ("k_hr2", c_vp), ("v_hr2", c_vp), ("kv_split", c_int)]


class WinattnTiling(ctypes.Structure):
    _fields_ = [("bw_q", c_int), ("bh_q", c_int), ("qboxes_per_tile", c_int),
                ("m_tiles", c_int), ("bw_k", c_int), ("bh_k", c_int),
                ("kboxes_per_tile", c_int), ("bw_a", c_int), ("bh_a", c_int),
                ("aboxes_per_tile", c_int), ("has_anchor", c_int), ("split_kv", c_int)]


SRDIT_EPI_PEER = 4
SRDIT_MAX_RANKS = 8
SRDIT_RED_SUM, SRDIT_RED_MAX = 0, 1
SRDIT_AR_BLOCKS = 16


class PeerPtrs(ctypes.Structure):
    _fields_ = [("p", c_vp * SRDIT_MAX_RANKS)]


class VRing(ctypes.Structure):
    _fields_ = [("ring", c_vp), ("ld", c_ll), ("col0", c_int), ("frame_tokens", c_int),
                ("slot0", c_int), ("n_slots", c_int)]


class TpGemm(ctypes.Structure):
    _fields_ = [("ag_flags", c_vp), ("ag_expected", ctypes.c_uint32),
                ("rows_per_rank", c_int), ("rank", c_int), ("world", c_int),
                ("rs_slot", c_vp * SRDIT_MAX_RANKS), ("ld_rs", c_ll),
                ("rs_flags", c_vp * SRDIT_MAX_RANKS), ("v_ring", ctypes.POINTER(VRing))]


class RopeHalo(ctypes.Structure):
    _fields_ = [("k", c_vp * 2), ("v", c_vp * 2), ("grid_w", c_int * 2), ("w0", c_int * 2),
                ("col_lo", c_int * 2), ("col_hi", c_int * 2), ("flag", c_vp * 2),
                ("done", c_vp)]


class DupUp(ctypes.Structure):
    _fields_ = [("x", c_vp), ("frames", c_int), ("cin", c_int), ("ft", c_int),
                ("repeats", c_int), ("shift", c_int)]


class Conv3dArgs(ctypes.Structure):
    _fields_ = [("x", c_vp), ("in_frames", c_int), ("out_frames", c_int), ("H", c_int),
                ("W", c_int), ("cin", c_int), ("kt", c_int), ("kh", c_int), ("weight", c_vp),
                ("bias", c_vp), ("cout", c_int), ("residual", c_vp), ("res_scale", c_float),
                ("relu", c_int), ("shuffle", c_int), ("shuffle_t", c_int),
                ("up2_phase", c_int), ("dup", ctypes.POINTER(DupUp)), ("out", c_vp),
                ("status", c_vp)]


# name -> argtypes (every function returns int)
SIGNATURES = {
    "srdit_version": [],
    "srdit_fp8_gemm": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int,
                       c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_vp],
    "srdit_quant_rowwise": [c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_ll, c_vp, c_vp],
    "srdit_ln_mod_quant": [c_vp, c_ll, c_int, c_int, c_float, c_vp, c_vp, c_vp, c_vp, c_vp,
                           c_ll, c_vp, c_vp],
    "srdit_rms_rope": [c_vp, c_ll, c_int, c_int, c_vp, c_float, c_vp, c_ll, c_int, c_int,
                       c_int, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_ll, c_vp, c_ll,
                       c_vp, c_int, c_vp, c_int, c_int, c_int, ctypes.POINTER(RopeHalo),
                       c_vp],
    "srdit_row_reduce": [c_vp, c_ll, c_int, c_int, c_int, c_vp, c_vp],
    "srdit_fp8_gemm_tp": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int,
                          c_int, c_int, c_vp, ctypes.POINTER(TpGemm), c_vp, c_vp],
    "srdit_fp8_gemm_ctas": [c_int, c_int],
    "srdit_fp8_gemm_vring": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int,
                             c_int, c_int, ctypes.POINTER(VRing), c_vp, c_vp],
    "srdit_residual_tp": [c_vp, c_ll, c_int, c_int, c_vp, c_int, c_ll, c_ll, c_vp, c_vp, c_vp,
                          ctypes.c_uint32, c_vp, c_vp],
    "srdit_tp_allreduce": [c_vp, c_vp, c_int, c_int, ctypes.POINTER(PeerPtrs),
                           ctypes.POINTER(PeerPtrs), c_int, c_int, ctypes.c_uint32, c_vp, c_vp],
    "srdit_ln_mod_quant_tp": [c_vp, c_ll, c_int, c_int, c_float, c_vp, c_vp, c_vp, c_vp, c_ll,
                              ctypes.POINTER(PeerPtrs), ctypes.POINTER(PeerPtrs),
                              ctypes.POINTER(PeerPtrs), c_vp, c_int, c_int, c_vp],
    "srdit_ln_mod_quant_tp_static": [c_vp, c_ll, c_int, c_int, c_float, c_vp, c_vp, c_vp, c_vp,
                                     c_ll, ctypes.POINTER(PeerPtrs), ctypes.POINTER(PeerPtrs),
                                     ctypes.POINTER(PeerPtrs), c_int, c_int, c_vp],
    "srdit_tp_push": [c_vp, ctypes.POINTER(PeerPtrs), ctypes.c_ulonglong, c_vp,
                      ctypes.POINTER(PeerPtrs), ctypes.c_ulonglong, ctypes.POINTER(PeerPtrs),
                      c_int, c_int, c_vp],
    "srdit_conv3x3": [c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_int,
                      c_vp, c_float, c_int, c_int, c_vp, c_vp, c_vp],
    "srdit_conv3d": [ctypes.POINTER(Conv3dArgs), c_vp],
    "srdit_rms_silu": [c_vp, c_ll, c_int, c_vp, c_int, c_vp, c_vp],
    "srdit_wait_counters": [c_vp, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp],
    "srdit_ipc_handle": [c_vp, c_vp, ctypes.POINTER(ctypes.c_ulonglong)],
    "srdit_ipc_open": [c_vp, ctypes.POINTER(c_vp)],
    "srdit_ipc_close": [c_vp],
    "srdit_residual": [c_vp, c_ll, c_int, c_int, c_vp, c_int, c_ll, c_ll, c_vp, c_vp, c_vp],
    "srdit_winattn_plan": [c_vp, c_int, c_int, c_int, ctypes.POINTER(WinattnTiling)],
    "srdit_winattn_fwd": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                          ctypes.POINTER(WinattnGeom), ctypes.POINTER(WinattnTiling), c_vp,
                          c_vp],
}


class SrditError(RuntimeError):
    pass


_lock = threading.Lock()
_lib = None


def header_symbols() -> list[str]:
    """Every entry point declared in include/srdit_b200.h."""
    import re
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(srdit_\w+)\(", text, re.M)))


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it is absent or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise SrditError(
                f"{LIB_PATH} is missing: build it with `python {PKG / 'build.py'}` "
                "(there is no fallback path).")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = c_int
        L.srdit_strerror.argtypes = [c_int]
        L.srdit_strerror.restype = ctypes.c_char_p
        _lib = L
        return L


def count(name: str, *args) -> int:
    """Call an entry point that returns a count (not a status)."""
    return int(getattr(lib(), name)(*args))


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().srdit_strerror(rc).decode()
        raise SrditError(f"{what} failed with code {rc}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
