"""Shared test inputs: the golden plan cases and the seeded attention inputs."""
from __future__ import annotations

import numpy as np
import torch

PLAN_NAMES = [
    "cfg1_8x8_r0", "cfg1_4x4_r3", "2k_4x4_r3_f3", "2k_4x4_r3_f6", "2k_4x4_r3_f12",
    "2k_4x4_r3_f12_frame", "2k_4x4_r3_f6_chunk", "2k_8x8_r0_f6", "2k_8x8_r0_f12_frame",
    "2k_4x4_r3_harvest", "odd_f5", "odd_frame", "native_anchor", "hist_rt1", "parallel_causal",
]
SPEC_KEYS = ("f_cur", "f_kv", "h", "w", "block_t", "bh", "bw", "rh", "rw", "hist", "rt",
             "chunk_frames", "streaming")
MODES = {0: None, 1: "chunk", 2: "frame"}


def spec_fields(g, name):
    vals = dict(zip(SPEC_KEYS, (int(x) for x in g[f"{name}.spec"])))
    for k in ("hist", "chunk_frames"):
        if vals[k] == -1:
            vals[k] = None
    vals["streaming"] = bool(vals["streaming"])
    ahw = tuple(int(x) for x in g[f"{name}.anchor_hw"])
    vals["anchor_hw"] = None if ahw == (-1, -1) else ahw
    return vals, MODES[int(g[f"{name}.mode"])]


def spec_from_golden(g, name, cls):
    vals, mode = spec_fields(g, name)
    return cls(**vals), mode


def config1_inputs():
    """seed 0, q,k,v ~ N(0,1) fp32 [1728, 24, 128], RoPE on q,k."""
    from oracle import numerics as onum
    torch.manual_seed(0)
    q = torch.randn(1, 1728, 24, 128)[0]
    k = torch.randn(1, 1728, 24, 128)[0]
    v = torch.randn(1, 1728, 24, 128)[0]
    freqs = onum.rope_freqs()
    return onum.rope_apply(q, (3, 18, 32), freqs), onum.rope_apply(k, (3, 18, 32), freqs), v


def stream_inputs():
    g = torch.Generator().manual_seed(1)
    f_cur, f_cache, h, w, n, d = 3, 3, 8, 12, 2, 128
    L = h * w
    names = ("q", "k", "v", "ck", "cv", "ak", "av")
    sizes = (f_cur, f_cur, f_cur, f_cache, f_cache, f_cur, f_cur)
    return {nm: torch.randn(1, s * L, n, d, generator=g)[0] for nm, s in zip(names, sizes)}


def bf16_from_bits(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16)


def vae_param(name: str, shape, index: int):
    """The seeded value of parameter ``name`` (its ``index`` in the sorted names)
    of the golden VAE decoder: RMS_norm gammas 1 + 0.2 N(0, 1), conv weights
    N(0, 1) / sqrt(fan_in), biases 0.05 N(0, 1); fp32, rounded to bf16 by the
    user. The fixture stores only the names and shapes."""
    import torch
    g = torch.Generator().manual_seed(1000 + index)
    t = torch.randn(*shape, generator=g)
    if name.endswith(".gamma"):
        return 1 + 0.2 * t
    if name.endswith(".bias"):
        return 0.05 * t
    fan_in = 1
    for d in shape[1:]:
        fan_in *= int(d)
    return t / fan_in ** 0.5


def vae_state_dict(g):
    """The golden VAE decoder's bf16 state dict, regenerated from the fixture's
    names and shapes."""
    import torch
    names = [str(n) for n in g["param_names"]]
    shapes = g["param_shapes"]
    ndims = g["param_ndims"]
    sd = {}
    for i, (n, shp, nd) in enumerate(zip(names, shapes, ndims)):
        shape = tuple(int(v) for v in shp[:int(nd)])
        sd[n] = vae_param(n, shape, i).to(torch.bfloat16)
    return sd
