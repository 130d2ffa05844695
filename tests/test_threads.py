"""Ops called from a host thread whose first CUDA call they are (the autograd engine runs
backward on its own thread): the tensor-map encode binds the device's primary context
instead of failing."""

import threading

import pytest


@pytest.mark.gpu
def test_ops_from_a_fresh_thread(cuda):
    import torch
    from mzoo_b200 import indexer, swa_attn
    q = torch.randn(1, 64, 16, 128, device=cuda).to(torch.bfloat16)
    kv = torch.randn(1, 64, 1, 128, device=cuda).to(torch.bfloat16)
    k = torch.randn(1, 32, 128, device=cuda).to(torch.bfloat16)
    w = torch.randn(1, 64, 16, device=cuda)
    ref = swa_attn.fwd(q, kv, window=16)[0], indexer.fwd(q, k, w, compress_ratio=2)
    torch.cuda.synchronize()
    out, errs = {}, []

    def worker():
        try:
            out["o"] = swa_attn.fwd(q, kv, window=16)[0]
            out["s"] = indexer.fwd(q, k, w, compress_ratio=2)
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert not errs, errs
    assert torch.equal(out["o"], ref[0]) and torch.equal(out["s"], ref[1])
