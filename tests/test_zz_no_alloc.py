"""srdit_ln_mod_quant_tp_static: the entry point that allocates nothing.

Its last-CTA counter is the library's own device array instead of a caller
buffer. On one GPU (world = 1: the rank's own gather buffer, no peer to
signal) two calls in a row must each produce the bytes that the entry point
with a caller-provided counter produces for the same rows -- which also shows
that the kernel leaves the static counter at 0 for the next call.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_static_counter_entry_matches_the_caller_buffer_entry(srdit, cuda_device):
    lib_mod = srdit._lib
    L = lib_mod.lib()
    M, K = 1000, 3072
    g = torch.Generator().manual_seed(21)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    outs = {}
    for name in ("srdit_ln_mod_quant_tp", "srdit_ln_mod_quant_tp_static"):
        res = []
        for call in range(2):
            x = (torch.randn(M, K, generator=g) * (1 + call)).to(torch.bfloat16).to(cuda_device)
            shift = (0.1 * torch.randn(K, generator=g)).to(cuda_device)
            scale = (0.1 * torch.randn(K, generator=g)).to(cuda_device)
            q = torch.zeros(M, K, dtype=torch.uint8, device=cuda_device)
            s = torch.zeros(M, dtype=torch.float32, device=cuda_device)
            flags = torch.zeros(8, dtype=torch.int32, device=cuda_device)
            qt, st, ft = lib_mod.PeerPtrs(), lib_mod.PeerPtrs(), lib_mod.PeerPtrs()
            qt.p[0], st.p[0], ft.p[0] = q.data_ptr(), s.data_ptr(), flags.data_ptr()
            args = [ctypes.c_void_p(x.data_ptr()), K, M, K, 1e-6, None, None,
                    ctypes.c_void_p(shift.data_ptr()), ctypes.c_void_p(scale.data_ptr()), K,
                    ctypes.byref(qt), ctypes.byref(st), ctypes.byref(ft)]
            if name == "srdit_ln_mod_quant_tp":
                done = torch.zeros(1, dtype=torch.int32, device=cuda_device)
                args.append(ctypes.c_void_p(done.data_ptr()))
            rc = getattr(L, name)(*args, 0, 1, stream)
            assert rc == 0, lib_mod.strerror(rc) if hasattr(lib_mod, "strerror") else rc
            torch.cuda.synchronize(cuda_device)
            res.append((q.cpu(), s.cpu()))
        outs[name] = res
        g = torch.Generator().manual_seed(21)   # the same rows for the other entry point
    for (qa, sa), (qb, sb) in zip(outs["srdit_ln_mod_quant_tp"],
                                  outs["srdit_ln_mod_quant_tp_static"]):
        assert torch.equal(qa, qb)
        assert torch.equal(sa, sb)
        assert bool((sa > 0).all())
