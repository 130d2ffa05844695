"""Every kernel is a ``torch.library`` custom op ``mzb::*`` with a fake implementation: the
ops trace (shape/dtype propagation on meta tensors) without a GPU or the library."""

import torch

import mzoo_b200.ops  # noqa: F401  (registers the ops)

M = dict(device="meta")


def test_all_ops_registered():
    names = {"fq_fp4", "fq_fp8", "indexer_scores", "indexer_topk", "indexer_bwd", "attn_fwd", "attn_bwd",
             "sparse_mla_fwd", "candidate_blocks", "candidate_topk", "compress", "norm_rope_fwd", "norm_rope_bwd"}
    assert names <= set(dir(torch.ops.mzb))


def test_fake_shapes():
    B, S, Hi, Di, T = 2, 64, 64, 128, 100
    q = torch.empty(B, S, Hi, Di, dtype=torch.float8_e4m3fn, **M)
    k = torch.empty(B, T, Di, dtype=torch.float8_e4m3fn, **M)
    w = torch.empty(B, S, Hi, dtype=torch.float32, **M)
    sc = torch.ops.mzb.indexer_scores(q, k, w, None, None, None, None, 4, 0, 1.0, 3, True, False)
    assert sc.shape == (B, S, T) and sc.dtype == torch.float32
    idx = torch.ops.mzb.indexer_topk(sc, q, k, w, None, None, None, None, 4, 0, 1.0, 3, 16, 2.0**-21, 16, False)
    kp = torch.empty(9, 64, Di, dtype=torch.float8_e4m3fn, **M)
    pt = torch.empty(B, 3, dtype=torch.int32, **M)
    assert torch.ops.mzb.indexer_scores(q, kp, w, None, None, None, pt, 4, 0, 1.0, 3, True, False).shape == (B, S, 192)
    assert idx.shape == (B, S, 16) and idx.dtype == torch.int32
    qb = torch.empty(B, S, Hi, Di, dtype=torch.bfloat16, **M)
    kb = torch.empty(B, T, Di, dtype=torch.bfloat16, **M)
    dq, dk, dw = torch.ops.mzb.indexer_bwd(qb, kb, w, sc, 4, 0, 0.1, False)
    assert dq.shape == qb.shape and dk.shape == kb.shape and dw.shape == w.shape
    H, D = 16, 128
    qa = torch.empty(B, S, H, D, dtype=torch.bfloat16, **M)
    kv = torch.empty(B, S, 1, D, dtype=torch.bfloat16, **M)
    o, lse = torch.ops.mzb.attn_fwd(qa, kv, None, None, None, None, 32, 0.1, False)
    assert o.shape == qa.shape and lse.shape == (B, S * H)
    g = torch.ops.mzb.attn_bwd(qa, kv, kv, None, None, o, lse, o, 32, 0.1, False)
    assert g[0].shape == qa.shape and g[1].shape == (B, S, 1, D) and g[2].shape == (B, S, 1, D)
    assert g[4].shape == (B, -(-S * H // 128) * 128)
    qm = torch.empty(10, 128, 576, dtype=torch.bfloat16, **M)
    rows = torch.empty(1, 50, 672, dtype=torch.uint8, **M)
    ii = torch.empty(10, 8, dtype=torch.int32, **M)
    pos = torch.empty(10, dtype=torch.int32, **M)
    om, lm = torch.ops.mzb.sparse_mla_fwd(qm, rows, rows, ii, pos, None, None, None, 10, 10, 8, 4, 50, 50, 0, 0, 0.04,
                                          False)
    assert om.shape == (10, 128, 512) and lm.shape == (10, 128)
    x = torch.empty(4, 64, dtype=torch.bfloat16, **M)
    assert torch.ops.mzb.fq_fp4(x, 32, 0).shape == x.shape and torch.ops.mzb.fq_fp8(x, 32, 0).shape == x.shape
    lg = torch.empty(12, 300, dtype=torch.float32, **M)
    cl = torch.empty(12, dtype=torch.int32, **M)
    blocks, mask = torch.ops.mzb.candidate_blocks(lg, cl, 16, 8, True)
    assert blocks.shape == (12, 16) and blocks.dtype == torch.int32
    assert mask.shape == (12, 300) and mask.dtype == torch.uint8
    assert torch.ops.mzb.candidate_blocks(lg, cl, 16, 8, False)[1].shape == (0,)
    top = torch.ops.mzb.candidate_topk(lg, blocks, None, 8, 24)
    assert top.shape == (12, 24) and top.dtype == torch.int32
    kv = torch.empty(2, 40, 576, dtype=torch.float32, **M)
    nw = torch.empty(576, dtype=torch.bfloat16, **M)
    cs = torch.empty(2, 10, 32, dtype=torch.float32, **M)
    lat, cache = torch.ops.mzb.compress(kv, kv, nw, cs, cs, 4, 64, 1e-6)
    assert lat.shape == (2, 10, 576) and cache.shape == (2, 10, 576) and lat.dtype == torch.bfloat16
    assert torch.ops.mzb.compress(kv, kv, nw, None, None, 4, 0, 1e-6)[1].shape == (0,)
    xr = torch.empty(64, 128, dtype=torch.bfloat16, **M)
    cs = torch.empty(16, 32, dtype=torch.float32, **M)
    out, rstd = torch.ops.mzb.norm_rope_fwd(xr, torch.empty(128, dtype=torch.bfloat16, **M), cs, cs, 4, 1e-6)
    assert out.shape == xr.shape and rstd.shape == (64,)
    dx, dw = torch.ops.mzb.norm_rope_bwd(xr, torch.empty(128, dtype=torch.bfloat16, **M), cs, cs, rstd, xr, 4)
    assert dx.shape == xr.shape and dw.shape == (128,) and dw.dtype == torch.float32
