"""576/512 FP8-latent sparse attention: prefill and paged decode against the CPU oracle.

Tolerance (north-star): outputs and lse within max-abs 2e-2 of the fp64 oracle on the
same packed rows.  Cases mirror the reference's csa2 test matrix
(``csa2_attn/fwd_test.py:82-195``): -1 padding, topk > visible, non-tile-aligned topk and
window, duplicate indices (counted twice), and a window-only degenerate case.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import mla as M
from oracle.quant import bf16_to_f32

ATOL = 2e-2


# ----------------------------------------------------------------------------- CPU

def test_oracle_rows_roundtrip():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((50, 576)).astype(np.float32)
    back = M.unpack_rows(M.pack_rows(x))
    rel = np.abs(back[:, :512] - x[:, :512]) / (np.abs(x[:, :512]).reshape(50, 8, 64).max(-1).repeat(64, 1) + 1e-9)
    assert rel.max() <= 2.0**-4  # e4m3 step relative to the tile scale
    assert np.abs(back[:, 512:] - x[:, 512:]).max() <= 2.0**-8 * np.abs(x[:, 512:]).max()


def test_oracle_attend_matches_dense_softmax():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((4, 576))
    k = rng.standard_normal((9, 576))
    o, lse = M.attend_rows(q, k, 0.1)
    z = q @ k.T * 0.1
    p = np.exp(z) / np.exp(z).sum(-1, keepdims=True)
    np.testing.assert_allclose(o, p @ k[:, :512], rtol=1e-12)
    np.testing.assert_allclose(lse, np.log(np.exp(z).sum(-1)), rtol=1e-12)


def _golden():
    return np.load(os.path.join(GOLDEN, "mla.npz"))


def test_oracle_pack_matches_reference_fixture():
    """The oracle's row packing (absmax/448 per 64 channels, e4m3 round to nearest even,
    bf16 rope) equals torch's float8_e4m3fn / bfloat16 casts bit for bit."""
    d = _golden()
    assert np.array_equal(M.pack_rows(d["pre.kv"]), d["pre.raw_rows"])
    assert np.array_equal(M.pack_rows(d["pre.cmp"]), d["pre.cmp_rows"])


def test_oracle_prefill_matches_reference_attend():
    """oracle.mla.sparse_prefill against the reference's ``_attend`` (golden_ref.py:83-100)
    on each query's gathered rows: window, duplicates counted twice, -1 and out-of-range
    slots empty, absolute positions (q_offset)."""
    d = _golden()
    q_offset, window = (int(x) for x in d["pre.params"])
    q = bf16_to_f32(d["pre.q"])[None]
    o, lse = M.sparse_prefill(q, d["pre.raw_rows"][None], d["pre.cmp_rows"][None], d["pre.idx"][None], window,
                              q_offset=q_offset)
    np.testing.assert_allclose(o[0], d["pre.o"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(lse[0], d["pre.lse"], rtol=0, atol=2e-5)


def test_oracle_decode_matches_reference_attend():
    """oracle.mla.sparse_decode (page tables, window over the last tokens, compressed entries
    below each sequence's compressed length) against the reference's ``_attend``."""
    d = _golden()
    window = int(d["dec.params"][0])
    o, lse = M.sparse_decode(bf16_to_f32(d["dec.q"]), d["dec.raw_pages"], d["dec.pt"], d["dec.lens"],
                             d["dec.cmp_pages"], d["dec.cpt"], d["dec.clens"], d["dec.idx"], window)
    np.testing.assert_allclose(o, d["dec.o"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(lse, d["dec.lse"], rtol=0, atol=2e-5)


# ----------------------------------------------------------------------------- GPU helpers

def _bf16(torch, x, dev):
    return torch.from_numpy(x).to(torch.bfloat16).to(dev)


def _prefill_case(torch, dev, B, S, G, topk, ratio, window, q_offset=0, dup=False, holes=False, seed=0):
    from mzoo_b200 import sparse_mla
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, S, 128, 576)).astype(np.float32)
    kv = rng.standard_normal((B, S + q_offset, 576)).astype(np.float32)
    cmp = rng.standard_normal((B, G, 576)).astype(np.float32)
    idx = np.full((B, S, topk), -1, np.int32)
    for b in range(B):
        for s in range(S):
            vis = min(G, (s + q_offset + 1) // ratio)
            sel = np.sort(rng.permutation(vis)[:topk]) if vis else np.zeros(0, np.int64)
            idx[b, s, :len(sel)] = sel
            if dup and len(sel) >= 2:
                idx[b, s, 1] = idx[b, s, 0]
            if holes and len(sel) >= 4:
                idx[b, s, 2] = -1
    qt = _bf16(torch, q, dev)
    raw_rows = sparse_mla.pack_kv(torch.from_numpy(kv).to(dev))
    cmp_rows = sparse_mla.pack_kv(torch.from_numpy(cmp).to(dev))
    o, lse = sparse_mla.prefill(qt, raw_rows, cmp_rows, torch.from_numpy(idx).to(dev), window=window,
                                q_offset=q_offset)
    qf = qt.float().cpu().numpy()
    ref_o, ref_lse = M.sparse_prefill(qf, raw_rows.cpu().numpy(), cmp_rows.cpu().numpy(), idx, window,
                                      q_offset=q_offset)
    return o.float().cpu().numpy(), lse.cpu().numpy(), ref_o, ref_lse


def _check(o, lse, ref_o, ref_lse, what):
    eo = np.abs(o - ref_o).max()
    el = np.abs(lse - ref_lse).max()
    print(f"{what}: max|o-ref|={eo:.3e} max|lse-ref|={el:.3e}")
    assert eo <= ATOL, f"{what}: o err {eo}"
    assert el <= ATOL, f"{what}: lse err {el}"


@pytest.mark.gpu
def test_prefill_basic(cuda):
    import torch
    r = _prefill_case(torch, cuda, B=1, S=192, G=48, topk=40, ratio=4, window=128)
    _check(*r, "prefill basic")


@pytest.mark.gpu
def test_prefill_ragged_dups_holes_offset(cuda):
    import torch
    r = _prefill_case(torch, cuda, B=2, S=130, G=70, topk=70, ratio=2, window=100, q_offset=5, dup=True, holes=True,
                      seed=3)
    _check(*r, "prefill ragged")


@pytest.mark.gpu
def test_prefill_window_only(cuda):
    """topk = 0 is the window-only (swa) degenerate case."""
    import torch
    r = _prefill_case(torch, cuda, B=1, S=100, G=16, topk=0, ratio=4, window=37, seed=5)
    _check(*r, "window only")


@pytest.mark.gpu
def test_decode_paged(cuda):
    import torch
    from mzoo_b200 import sparse_mla
    rng = np.random.default_rng(9)
    B, topk, window, ratio = 6, 128, 128, 4
    lens = rng.integers(100, 3000, B)
    max_pages = int(-(-lens.max() // 64))
    n_pages = B * max_pages
    perm = rng.permutation(n_pages).astype(np.int32)
    pt = perm.reshape(B, max_pages)
    cmp_lens = (lens // ratio).astype(np.int32)
    max_cp = int(-(-cmp_lens.max() // 64))
    cperm = rng.permutation(B * max_cp).astype(np.int32)
    cpt = cperm.reshape(B, max_cp)
    raw = rng.standard_normal((n_pages, 64, 576)).astype(np.float32)
    cmp = rng.standard_normal((B * max_cp, 64, 576)).astype(np.float32)
    idx = np.full((B, topk), -1, np.int32)
    for b in range(B):
        sel = np.sort(rng.permutation(int(cmp_lens[b]))[:topk])
        idx[b, :len(sel)] = sel
    q = rng.standard_normal((B, 128, 576)).astype(np.float32)
    raw_rows = sparse_mla.pack_kv(torch.from_numpy(raw).to(cuda))
    cmp_rows = sparse_mla.pack_kv(torch.from_numpy(cmp).to(cuda))
    qt = _bf16(torch, q, cuda)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)  # noqa: E731
    o, lse = sparse_mla.decode(qt, raw_rows, t(pt), t(lens.astype(np.int32)), cmp_rows, t(cpt), t(cmp_lens), t(idx),
                               window=window)
    ref_o, ref_lse = M.sparse_decode(qt.float().cpu().numpy(), raw_rows.cpu().numpy(), pt, lens,
                                     cmp_rows.cpu().numpy(), cpt, cmp_lens, idx, window)
    _check(o.float().cpu().numpy(), lse.cpu().numpy(), ref_o, ref_lse, "decode paged")


@pytest.mark.gpu
def test_prefill_deterministic(cuda):
    """No atomics in the forward: two runs are bit-identical."""
    import torch
    from mzoo_b200 import sparse_mla
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(1, 64, 128, 576, generator=g).to(torch.bfloat16).to(cuda)
    kv = sparse_mla.pack_kv(torch.randn(1, 64, 576, generator=g).to(cuda))
    cmp = sparse_mla.pack_kv(torch.randn(1, 16, 576, generator=g).to(cuda))
    idx = torch.randint(0, 16, (1, 64, 24), generator=g, dtype=torch.int32).to(cuda)
    a = sparse_mla.prefill(q, kv, cmp, idx)
    b = sparse_mla.prefill(q, kv, cmp, idx)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.gpu
def test_prefill_token_shards_match_full(cuda):
    """One rank's cyclic shard of query tokens (explicit q_pos) reproduces the rows of the
    full prefill: every token's attention is independent of the others.  (A shard with few
    tokens may run as key-range splits merged by the combine kernel, so the comparison is
    to rounding, not bitwise.)"""
    import torch
    from mzoo_b200 import sparse_mla
    from mzoo_b200.sharding import shard_tokens
    rng = np.random.default_rng(11)
    B, S, G, topk, window = 1, 256, 64, 32, 64
    q = torch.from_numpy(rng.standard_normal((B, S, 128, 576)).astype(np.float32)).to(torch.bfloat16).to(cuda)
    raw = sparse_mla.pack_kv(torch.from_numpy(rng.standard_normal((B, S, 576)).astype(np.float32)).to(cuda))
    cmp = sparse_mla.pack_kv(torch.from_numpy(rng.standard_normal((B, G, 576)).astype(np.float32)).to(cuda))
    idx = np.full((B, S, topk), -1, np.int32)
    for s in range(S):
        n = min(G, (s + 1) // 4)
        sel = np.sort(rng.permutation(n)[:topk])
        idx[0, s, :len(sel)] = sel
    it = torch.from_numpy(idx).to(cuda)
    o, lse = sparse_mla.prefill(q, raw, cmp, it, window=window)
    for part in shard_tokens(S, 3, chunk=32):
        tk = torch.tensor(part, device=cuda)
        os_, ls_ = sparse_mla.prefill(q[:, tk], raw, cmp, it[:, tk], window=window, q_pos=tk.view(1, -1))
        assert (os_.float() - o[:, tk].float()).abs().max() <= 1e-2
        assert (ls_ - lse[:, :, tk]).abs().max() <= 1e-3


@pytest.mark.gpu
def test_prefill_few_tokens_key_splits(cuda):
    """Few query tokens (fewer than half the SM pairs): each token's key list runs as
    several key-range splits merged by the combine kernel, including splits left empty."""
    import torch
    r = _prefill_case(torch, cuda, B=1, S=12, G=40, topk=40, ratio=1, window=100, q_offset=150, seed=8)
    _check(*r, "prefill few tokens")
