"""The drop-in wrappers never block the host on their default path (the reference's
wrappers do not): no ``Tensor.item`` / ``int(tensor)`` / ``tolist`` and no device
synchronisation.  Runs on the CPU: the wrappers trace under ``FakeTensorMode`` with fake
CUDA tensors, where every op dispatches to its fake implementation."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from mzoo_b200 import csa2_attn, indexer, norm_rope, ops, quant, sparse_mla, swa_attn

# ops whose last argument asks for an error-word read (a host synchronisation) after the launch
CHECKED_OPS = ("indexer_scores", "indexer_topk", "indexer_bwd", "attn_fwd", "attn_bwd", "sparse_mla_fwd")


def _forbid(monkeypatch):
    def boom(*a, **k):
        raise AssertionError("host synchronisation on the default path")
    for name in ("item", "tolist", "__int__", "__float__", "__index__"):
        monkeypatch.setattr(torch.Tensor, name, boom)
    monkeypatch.setattr(torch.cuda, "synchronize", boom)
    for name in CHECKED_OPS:  # the op itself reads its error word only when check=True
        op = getattr(ops, name)

        def no_check(*args, _op=op, _name=name):
            assert args[-1] is False, f"{_name} launched with check=True on the default path"
            return _op(*args)
        monkeypatch.setattr(ops, name, no_check)


@pytest.fixture
def fake(monkeypatch):
    with FakeTensorMode():
        _forbid(monkeypatch)
        yield torch.device("cuda", 0)


def test_indexer_wrappers_do_not_sync(fake):
    B, S, Hi, Di, T = 2, 64, 64, 128, 32
    q = torch.empty(B, S, Hi, Di, device=fake, dtype=torch.float8_e4m3fn)
    k = torch.empty(B, T, Di, device=fake, dtype=torch.float8_e4m3fn)
    w = torch.empty(B, S, Hi, device=fake)
    sq, sk = torch.empty(B, S, Hi, device=fake), torch.empty(B, T, device=fake)
    pos = torch.empty(B, S, device=fake, dtype=torch.int32)
    assert indexer.attn(q, k, w, compress_ratio=4, topk=16, scales=(sq, sk), q_pos=pos).shape == (B, S, 16)
    assert indexer.fwd(q, k, w, compress_ratio=4, scales=(sq, sk)).shape == (B, S, T)
    qb = torch.empty(B, S, Hi, Di, device=fake, dtype=torch.bfloat16)
    kb = torch.empty(B, T, Di, device=fake, dtype=torch.bfloat16)
    dl = torch.empty(B, S, T, device=fake)
    assert indexer.bwd(qb, kb, w, dl, compress_ratio=4)[0].shape == qb.shape


def test_attention_wrappers_do_not_sync(fake):
    B, S, H, D, G = 1, 64, 16, 128, 16
    q = torch.empty(B, S, H, D, device=fake, dtype=torch.bfloat16)
    kv = torch.empty(B, S, 1, D, device=fake, dtype=torch.bfloat16)
    o, lse = swa_attn.fwd(q, kv, window=32)
    swa_attn.bwd(q, kv, o, lse, o, window=32, causal=True, sinks=None)
    main = torch.empty(B, G, 1, D, device=fake, dtype=torch.bfloat16)
    idx = torch.empty(B, S, 8, device=fake, dtype=torch.int32)
    o, lse = csa2_attn.fwd(q, kv, main, idx, window=32, compress_ratio=4)
    csa2_attn.bwd(q, kv, main, idx, o, lse, o, window=32, compress_ratio=4)


def test_sparse_mla_wrappers_do_not_sync(fake):
    S, G = 32, 8
    q = torch.empty(1, S, 128, 576, device=fake, dtype=torch.bfloat16)
    rows = torch.empty(1, S, 672, device=fake, dtype=torch.uint8)
    crows = torch.empty(1, G, 672, device=fake, dtype=torch.uint8)
    idx = torch.empty(1, S, 16, device=fake, dtype=torch.int32)
    pos = torch.empty(1, S, device=fake, dtype=torch.int32)
    assert sparse_mla.prefill(q, rows, crows, idx, q_pos=pos)[0].shape == (1, S, 128, 512)
    B = 4
    qd = torch.empty(B, 128, 576, device=fake, dtype=torch.bfloat16)
    pages = torch.empty(10, 64, 672, device=fake, dtype=torch.uint8)
    pt = torch.empty(B, 3, device=fake, dtype=torch.int32)
    lens = torch.empty(B, device=fake, dtype=torch.int32)
    didx = torch.empty(B, 16, device=fake, dtype=torch.int32)
    assert sparse_mla.decode(qd, pages, pt, lens, pages, pt, lens, didx)[0].shape == (B, 128, 512)


def test_quant_wrappers_do_not_sync(fake):
    x = torch.empty(8, 128, device=fake, dtype=torch.bfloat16)
    quant._fake_quant_fp4_block(x, 32)
    quant._fake_quant_fp8_block(x, 32)


def test_norm_rope_does_not_sync(fake):
    x = torch.empty(1, 16, 4, 128, device=fake, dtype=torch.bfloat16)
    w = torch.empty(128, device=fake, dtype=torch.bfloat16)
    cs = torch.empty(1, 16, 32, device=fake)
    out, rstd = norm_rope.fwd(x, w, cs, cs)
    dx, dw = norm_rope.bwd(x, w, cs, cs, rstd, out)
    assert dx.shape == x.shape and dw.shape == (128,)
