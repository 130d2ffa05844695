"""Parity at the BASELINE configs' full sizes (the workloads ``bench.py`` times, built by the
bench's own input generators): every output row is checked for the size-independent
properties (ascending distinct in-range indices, finite outputs), and a sample of rows
against the CPU oracle -- bit-exact index sets for the indexer, max-abs 2e-2 for attention
outputs and lse.

- C2: B=2, 4096 queries at positions 12288..16383 x 4096 compressed keys, Hi=64, Di=128,
  FP8, top-512: 256 sampled query rows (four 64-row chunks over both batches).
- C3: 16384 tokens x 128 heads, top-2048 compressed + 128-token window: 32 sampled tokens.
- C4: 128 sequences with lengths in [8192, 131072], paged FP8 latent caches and index keys
  (64-key pages), decode indexer top-2048 + window 128: 8 sampled sequences (indexer sets
  and attention).
- C5: B=4, S=8192, 64 heads, D=128, window 512, after the MXFP4 / FP8 fake quant: dK / dV
  of three 128-key tiles (first, middle, last) and dQ of the tokens beside them, against the
  oracle's backward over the tokens those rows depend on; max-abs within 2e-2 + 1e-2 x the
  tensor's largest magnitude (the gradient tolerance of the attention tests).
"""

import numpy as np
import pytest

import bench
from oracle import attention as A
from oracle import indexer as I
from oracle import mla as M

ATOL = 2e-2
GRAD_RTOL = 1e-2


def _check_index_rows(idx: np.ndarray, vis: np.ndarray, topk: int) -> None:
    """Every row: ascending, distinct, in [0, vis), exactly min(topk, vis) entries, -1 after."""
    n = (idx >= 0).sum(-1)
    assert np.array_equal(n, np.minimum(topk, vis)), "wrong number of selected keys"
    first_pad = np.where(idx < 0, 1, 0).argmax(-1)
    ok_pad = np.where(n < topk, first_pad == n, True)
    assert ok_pad.all(), "-1 padding not at the end"
    d = np.diff(np.where(idx < 0, np.iinfo(np.int32).max, idx), axis=-1)
    assert (d > 0).all(), "indices not strictly ascending"
    assert (idx.max(-1) < vis).all(), "index beyond the visible range"


@pytest.mark.gpu
def test_c2_indexer_full_size(cuda):
    import torch
    from mzoo_b200 import indexer
    C2 = bench.C2
    q, k, w = bench.c2_inputs(torch, seed=0)
    q8, sq = indexer.quantize_fp8(q.to(cuda))
    k8, sk = indexer.quantize_fp8(k.to(cuda))
    wd = w.to(cuda)
    got = indexer.attn(q8, k8, wd, compress_ratio=C2["ratio"], topk=C2["topk"], q_offset=C2["q_offset"],
                       scales=(sq, sk), check=True).cpu().numpy()
    B, S, T = C2["B"], C2["S"], C2["T"]
    vis = np.minimum(T, (C2["q_offset"] + np.arange(S) + 1) // C2["ratio"])
    _check_index_rows(got, np.broadcast_to(vis, (B, S)), C2["topk"])
    qv, kv = q8.float().cpu().numpy(), k8.float().cpu().numpy()
    sqn, skn, wn = sq.cpu().numpy(), sk.cpu().numpy(), w.numpy()
    for b, s0 in ((0, 0), (0, 2048), (1, 1000), (1, S - 64)):
        s1 = s0 + 64
        off = C2["q_offset"] + s0
        canon = I.canonical_scores(qv[b:b + 1, s0:s1], kv[b:b + 1], wn[b:b + 1, s0:s1], sqn[b:b + 1, s0:s1],
                                   skn[b:b + 1], C2["ratio"], off)
        ref = I.canonical_topk(canon, C2["topk"], C2["ratio"], off)
        assert np.array_equal(got[b:b + 1, s0:s1], ref), (b, s0)


@pytest.mark.gpu
def test_c3_prefill_full_size(cuda):
    import torch
    from mzoo_b200 import sparse_mla
    C3 = bench.C3
    q, raw, cmp, idx = bench.c3_inputs(torch, cuda, seed=0)
    o, lse = sparse_mla.prefill(q, raw, cmp, idx, window=C3["window"], check=True)
    assert torch.isfinite(lse).all() and not torch.isnan(o).any()
    S = C3["S"]
    toks = [0, 1, 3, 127, 128, 4095, 4096, 8191] + [int(t) for t in np.linspace(200, S - 1, 24)]
    raw_h, cmp_h = raw[0].cpu().numpy(), cmp[0].cpu().numpy()
    idx_h = idx[0].cpu().numpy()
    tk = torch.tensor(toks, device=cuda)
    qs = q[0, tk].float().cpu().numpy()
    os_, ls_ = o[0, tk].float().cpu().numpy(), lse[0, :, tk].cpu().numpy()
    for i, t in enumerate(toks):
        keys = M.unpack_rows(M.token_keys(raw_h, cmp_h, idx_h[t], t, C3["window"]))
        ro, rl = M.attend_rows(qs[i], keys, 576**-0.5)
        eo, el = np.abs(os_[i] - ro).max(), np.abs(ls_[:, i] - rl).max()
        assert eo <= ATOL and el <= ATOL, (t, eo, el)


@pytest.mark.gpu
def test_c4_decode_full_size(cuda):
    import torch
    from mzoo_b200 import indexer, sparse_mla
    C4 = bench.C4
    lens = bench.c4_lens(torch)
    seqs = list(range(C4["B"]))
    x = bench.c4_inputs(torch, cuda, seqs, lens)
    idx = indexer.attn(x["q8"], x["k8"], x["w"], compress_ratio=C4["ratio"], topk=C4["topk"],
                       scales=(x["sq"], x["sk"]), q_pos=x["pos"], k_page_table=x["cpt"], check=True)
    o, lse = sparse_mla.decode(x["q"], x["raw"], x["pt"], x["lens"], x["cmp"], x["cpt"], x["cmp_lens"], idx[:, 0],
                               window=C4["window"], check=True)
    idx_h = idx[:, 0].cpu().numpy()
    L = lens.numpy()
    _check_index_rows(idx_h, L // C4["ratio"], C4["topk"])
    assert torch.isfinite(lse).all() and not torch.isnan(o).any()
    order = np.argsort(L)
    sample = sorted({int(order[0]), int(order[-1]), *[int(order[i]) for i in (16, 40, 64, 90, 110)], 0})
    for b in sample:
        T = int(L[b]) // C4["ratio"]
        pages = x["cpt"][b, :-(-T // 64)].long()  # the index keys share the compressed cache's pages
        qv = x["q8"][b:b + 1].float().cpu().numpy()
        kv = x["k8"][pages].reshape(1, -1, C4["Di"])[:, :T].float().cpu().numpy()
        skv = x["sk"][pages].reshape(1, -1)[:, :T].cpu().numpy()
        canon = I.canonical_scores(qv, kv, x["w"][b:b + 1].cpu().numpy(), x["sq"][b:b + 1].cpu().numpy(), skv,
                                   C4["ratio"], int(L[b]) - 1)
        ref_idx = I.canonical_topk(canon, C4["topk"], C4["ratio"], int(L[b]) - 1)[0, 0]
        assert np.array_equal(idx_h[b], ref_idx), b
        # attention over the window + selected rows, gathered through the page tables on the GPU
        pos = torch.arange(max(0, int(L[b]) - C4["window"]), int(L[b]), device=cuda)
        sel = idx[b, 0][idx[b, 0] >= 0].long()
        rows = torch.cat([x["raw"][x["pt"][b, pos // 64].long(), pos % 64],
                          x["cmp"][x["cpt"][b, sel // 64].long(), sel % 64]])
        ro, rl = M.attend_rows(x["q"][b].float().cpu().numpy(), M.unpack_rows(rows.cpu().numpy()), 576**-0.5)
        eo = np.abs(o[b].float().cpu().numpy() - ro).max()
        el = np.abs(lse[b].cpu().numpy() - rl).max()
        assert eo <= ATOL and el <= ATOL, (b, eo, el)


@pytest.mark.gpu
def test_c5_train_full_size(cuda):
    import torch
    C5 = bench.C5
    B, S, H, D, W = (C5[x] for x in ("B", "S", "H", "D", "window"))
    g = torch.Generator(device=cuda).manual_seed(10)  # bench_train's inputs at rank 0
    q = torch.randn(B, S, H, D, generator=g, device=cuda, dtype=torch.bfloat16)
    k = torch.randn(B, S, 1, D, generator=g, device=cuda, dtype=torch.bfloat16)
    v = torch.randn(B, S, 1, D, generator=g, device=cuda, dtype=torch.bfloat16)
    do = torch.randn(B, S, H, D, generator=g, device=cuda, dtype=torch.bfloat16)
    dq, dk, dv = bench.c5_step(q, k, v, do)
    torch.cuda.synchronize()
    assert all(torch.isfinite(x).all() for x in (dq, dk, dv))
    from mzoo_b200 import quant
    qf = quant.fake_quant_fp4_block(q, 32, rule="ocp")
    kf = quant.fake_quant_fp4_block(k, 32, rule="ocp")
    vf = quant.fake_quant_fp8_block(v, 128, rule="absmax")

    def host(x, b, lo, hi):
        return x[b:b + 1, lo:hi].float().cpu().numpy()

    for b, j0 in ((0, 0), (1, 4096), (3, S - 128)):
        # keys [j0, j0 + 128) are seen by queries [j0, j0 + 128 + W - 1), whose windows start at
        # j0 - W + 1 or later: the oracle's backward over that slice is exact for them
        lo, hi = max(0, j0 - W + 1), min(S, j0 + 128 + W - 1)
        ref = A.attend_bwd(host(qf, b, lo, hi), host(kf, b, lo, hi)[:, :, 0], host(do, b, lo, hi), window=W,
                           v=host(vf, b, lo, hi)[:, :, 0])
        sl = slice(j0 - lo, j0 - lo + 128)
        for name, got, want in (("dk", dk[b, j0:j0 + 128, 0], ref["dk"][0, sl]),
                                ("dv", dv[b, j0:j0 + 128, 0], ref["dv"][0, sl]),
                                ("dq", dq[b, j0:j0 + 128], ref["dq"][0, sl])):
            err = np.abs(got.float().cpu().numpy() - want).max()
            tol = ATOL + GRAD_RTOL * np.abs(want).max()
            assert err <= tol, (name, b, j0, err, tol)
