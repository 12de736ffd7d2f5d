"""Host logic of the drop-in window-attention op (no GPU).

The op hands the kernel the cached frames and the current chunk as two K/V
segments, so it never concatenates them for the attention. The cache it
returns must still be what the reference returns: the last ``kv_len`` frames
of ``cat([cache, chunk])``, or all of them when ``kv_len`` is None
(attention.py:964-974).
"""
import importlib

import pytest
import torch

attention = importlib.import_module("dreamx-creator_b200.attention")

L, N, D = 6, 2, 4   # tokens per frame, heads, head dim


def _frames(f, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(f * L, N, D, generator=g)


@pytest.mark.parametrize("f_cache", [0, 1, 3, 9])
@pytest.mark.parametrize("f_cur", [1, 3])
@pytest.mark.parametrize("kv_len", [None, 1, 2, 3, 4, 9, 20])
def test_new_cache_is_the_reference_tail(f_cache, f_cur, kv_len):
    ck, cv = (_frames(f_cache, 1), _frames(f_cache, 2)) if f_cache else (None, None)
    k, v = _frames(f_cur, 3), _frames(f_cur, 4)
    nk, nv = attention._new_cache(ck, cv, k, v, kv_len, L)
    full_k = torch.cat([ck, k]) if ck is not None else k
    full_v = torch.cat([cv, v]) if cv is not None else v
    keep = full_k.shape[0] if kv_len is None else min(full_k.shape[0], kv_len * L)
    assert torch.equal(nk, full_k[full_k.shape[0] - keep:])
    assert torch.equal(nv, full_v[full_v.shape[0] - keep:])


def test_new_cache_is_a_view_when_the_chunk_covers_it():
    ck, cv = _frames(3, 1), _frames(3, 2)
    k, v = _frames(3, 3), _frames(3, 4)
    nk, nv = attention._new_cache(ck, cv, k, v, 2, L)
    assert nk.data_ptr() == k[L:].data_ptr() and nv.data_ptr() == v[L:].data_ptr()
