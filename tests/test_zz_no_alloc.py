"""The allocation-free sparse-attention entry point, called through the C ABI.

`mzb_sparse_mla_fwd_noalloc` serves callers that cannot allocate device memory when they
launch attention (a serving engine whose free HBM is all handed to its KV-cache pool, or a
host with its own memory manager): it takes its per-token workspace from a fixed array in
the library instead of from the caller.  Its results must match `mzb_sparse_mla_fwd`
(same kernel; this checks they are bit-identical, which is inside every tolerance the
attention tests use) on two calls in a row, the second reusing the scratch the first
left behind, and it must reject sizes beyond its fixed 65536-token scratch.

This file is named to be collected last, so a run that stops at its first failure has
already run every other test.
"""

import ctypes

import numpy as np
import pytest


def _inputs(torch, dev, S, G, topk, seed):
    from mzoo_b200 import sparse_mla
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(1, S, 128, 576, generator=g).to(torch.bfloat16).to(dev)
    raw = sparse_mla.pack_kv(torch.randn(1, S, 576, generator=g).to(dev))
    cmp = sparse_mla.pack_kv(torch.randn(1, G, 576, generator=g).to(dev))
    rng = np.random.default_rng(seed)
    idx = np.full((1, S, topk), -1, np.int32)
    for s in range(S):
        vis = min(G, (s + 1) // 4)
        sel = np.sort(rng.permutation(vis)[:topk]) if vis else []
        idx[0, s, :len(sel)] = sel
    pos = torch.arange(S, dtype=torch.int32, device=dev)
    return q, raw, cmp, torch.from_numpy(idx).to(dev), pos


def _call(torch, name, q, raw, cmp, idx, pos, S, G, topk, window=128):
    from mzoo_b200 import _lib
    lib = _lib.lib()
    dev = q.device
    o = torch.empty(S, 128, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(S, 128, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    common_head = [p(q), p(raw), p(cmp), p(idx), p(pos), None, None, None]
    head = [p(o), p(lse), S, S, topk, window, S, G, 0, 0, ctypes.c_float(576**-0.5)]
    tail = [p(err), stream]
    if name == "mzb_sparse_mla_fwd":  # one key-range split, like the allocation-free entry point
        slots = torch.empty(S, dtype=torch.int32, device=dev)
        status = lib.mzb_sparse_mla_fwd(*common_head, p(slots), *head, 1, None, *tail)
    else:
        status = lib.mzb_sparse_mla_fwd_noalloc(*common_head, *head, *tail)
    assert status == 0, lib.mzb_last_error()
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    return o, lse


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda):
    import torch
    for S, G, topk, seed in ((160, 40, 32, 0), (96, 24, 16, 1)):
        q, raw, cmp, idx, pos = _inputs(torch, cuda, S, G, topk, seed)
        o_ref, lse_ref = _call(torch, "mzb_sparse_mla_fwd", q, raw, cmp, idx, pos, S, G, topk)
        o, lse = _call(torch, "mzb_sparse_mla_fwd_noalloc", q, raw, cmp, idx, pos, S, G, topk)
        assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)


@pytest.mark.gpu
def test_noalloc_rejects_oversized_call(cuda):
    from mzoo_b200 import _lib
    lib = _lib.lib()
    status = lib.mzb_sparse_mla_fwd_noalloc(None, None, None, None, None, None, None, None, None, None, 65537, 1, 0,
                                           128, 1, 0, 0, 0, ctypes.c_float(1.0), None, None)
    assert status == _lib.MZB_ERR_SHAPE
    assert b"65536" in lib.mzb_last_error()
