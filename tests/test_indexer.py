"""Lightning indexer: oracle pinned to the reference's golden vectors (CPU); the sm_100a
score kernel against the oracle within the reference's acceptance criterion and with an
exactly equal -inf mask; top-k index sets bit-exact against the canonical oracle (GPU).

Reference tests mirrored: ``indexer/fwd_test.py:52-83`` (Hi x Di matrix, ratios,
non-aligned / empty T), ``indexer/attn_test.py:28-46`` (per-row set equality, topk > T
padding).
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import indexer as I
from oracle import quant as Q


def _golden():
    return np.load(os.path.join(GOLDEN, "indexer.npz"))


# ----------------------------------------------------------------------------- CPU: oracle pin

def test_oracle_scores_match_reference_golden():
    d = _golden()
    got = I.scores_ref(d["q"], d["k"], d["w"], 2)
    ref = d["scores"]
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    np.testing.assert_allclose(got[fin], ref[fin], rtol=0, atol=1e-5)


@pytest.mark.parametrize("topk", [4, 16, 25])
def test_oracle_topk_matches_reference_golden(topk):
    d = _golden()
    ref = np.sort(np.where(d[f"topk{topk}"] < 0, 1 << 30, d[f"topk{topk}"]), -1)
    ref = np.where(ref == 1 << 30, -1, ref)
    assert np.array_equal(I.topk_ref(d["scores"], topk), ref)


def test_canonical_topk_equals_reference_sets():
    """The canonical fp64 definition selects the same sets as the reference's fp32 path
    on its golden inputs (no near-ties there)."""
    d = _golden()
    q, k, w = d["q"], d["k"], d["w"]
    c = I.canonical_scores(q, k, w, None, None, 2, 0, scale=float(np.float32(q.shape[-1] ** -0.5)), fp8=False)
    for topk in (4, 16, 25):
        ref = I.topk_ref(d["scores"], topk)
        assert np.array_equal(I.canonical_topk(c, topk, 2), ref.astype(np.int32))


def _golden_fp8():
    return np.load(os.path.join(GOLDEN, "indexer_fp8.npz"))


def test_oracle_fp8_quantiser_matches_reference_fixture():
    """The oracle's absmax e4m3 quantiser equals torch's float8_e4m3fn cast (codes, scales)."""
    from oracle import mla as M
    d = _golden_fp8()
    di = d["q"].shape[-1]
    for x, codes, sc in ((d["q"], d["q_codes"], d["sq"]), (d["k"], d["k_codes"], d["sk"])):
        v, s = Q.quantize_fp8_rows(x, di)
        assert np.array_equal(s[..., 0], sc)
        assert np.array_equal(v, M.e4m3_values(codes))


def test_oracle_fp8_scores_and_sets_match_reference():
    """FP8 indexer numerics: the reference's fp32 ``indexer_scores`` on the dequantised
    q * s_q, k * s_k (golden_ref.py:213-227) equals the oracle's, and the canonical exact
    definition the kernel selects against (scale = Di**-0.5) picks the reference's sets."""
    from oracle import mla as M
    d = _golden_fp8()
    ratio = int(d["params"][0])
    qv, kv = M.e4m3_values(d["q_codes"]), M.e4m3_values(d["k_codes"])
    di = qv.shape[-1]
    qd = (qv * d["sq"][..., None]).astype(np.float32)
    kd = (kv * d["sk"][..., None]).astype(np.float32)
    got = I.scores_ref(qd, kd, d["w"], ratio)
    ref = d["scores"]
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    np.testing.assert_allclose(got[fin], ref[fin], rtol=0, atol=1e-5)
    canon = I.canonical_scores(qv, kv, d["w"], d["sq"], d["sk"], ratio, 0, scale=float(np.float32(di**-0.5)))
    for topk in (5, 12, 30):
        r = np.sort(np.where(d[f"topk{topk}"] < 0, 1 << 30, d[f"topk{topk}"]), -1)
        r = np.where(r == 1 << 30, -1, r)
        assert np.array_equal(I.canonical_topk(canon, topk, ratio), r.astype(np.int32)), topk


def test_canonical_fp8_dot_is_order_independent():
    """e4m3 products are multiples of 2^-18 below 2^17.6: any fp64 summation order is exact."""
    rng = np.random.default_rng(0)
    codes, _ = Q.quantize_fp8_rows(rng.standard_normal((64, 128)).astype(np.float32), 128)
    kc, _ = Q.quantize_fp8_rows(rng.standard_normal((32, 128)).astype(np.float32), 128)
    a = codes.astype(np.float64) @ kc.astype(np.float64).T
    b = np.zeros_like(a)
    for i in range(127, -1, -1):
        b = b + codes[:, None, i].astype(np.float64) * kc[None, :, i].astype(np.float64)
    assert np.array_equal(a, b)


def _e4m3_int(c: int) -> int:
    """The top-k kernel's integer form of an e4m3 code (``e4m3_int`` in csrc/indexer.cu):
    value = (M << (e' - 1)) * 2^-9, M = 8 + m (normal) or m (subnormal), e' = max(e, 1)."""
    e, m = (c >> 3) & 15, c & 7
    v = ((8 | m) if e else m) << ((e - 1) if e else 0)
    return -v if c & 0x80 else v


def test_e4m3_integer_dot_is_exact():
    """The wide top-k blocks re-score e4m3 band keys as int64 dot products in units of
    2^-18: every non-NaN code's integer form is its value x 2^9, and a 128-term integer dot
    (below 2^43) times 2^-18 equals the exact fp64 sum the canonical score defines."""
    import torch
    codes = np.arange(256, dtype=np.uint8)
    nan = (codes & 0x7F) == 0x7F
    vals = torch.from_numpy(codes).view(torch.float8_e4m3fn).double().numpy()
    ints = np.array([_e4m3_int(int(c)) for c in codes], dtype=np.int64)
    assert np.array_equal(ints[~nan].astype(np.float64) * 2.0**-9, vals[~nan])
    assert np.abs(ints[~nan]).max() < 2**18
    rng = np.random.default_rng(1)
    ok = codes[~nan]
    q = rng.choice(ok, size=(64, 128))
    k = rng.choice(ok, size=(16, 128))
    k[0] = 0x7E  # the largest codes: the bound's edge
    q[0] = 0x7E
    qi, ki = ints[q], ints[k]
    qv = torch.from_numpy(q).view(torch.float8_e4m3fn).double().numpy()
    kv = torch.from_numpy(k).view(torch.float8_e4m3fn).double().numpy()
    dot_int = qi @ ki.T  # int64, exact
    assert np.abs(dot_int).max() < 2**43
    assert np.array_equal(dot_int.astype(np.float64) * 2.0**-18, qv @ kv.T)


# ----------------------------------------------------------------------------- GPU

def _bf16_inputs(torch, dev, B, S, Hi, Di, T, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, S, Hi, Di, generator=g).to(torch.bfloat16)
    k = torch.randn(B, T, Di, generator=g).to(torch.bfloat16)
    w = torch.randn(B, S, Hi, generator=g) * Hi**-0.5
    return q.to(dev), k.to(dev), w.to(dev)


def _check_scores(torch, dev, B, S, Hi, Di, T, ratio, q_offset=0):
    from mzoo_b200 import indexer
    q, k, w = _bf16_inputs(torch, dev, B, S, Hi, Di, T)
    got = indexer.fwd(q, k, w, compress_ratio=ratio, q_offset=q_offset).cpu().numpy()
    qf, kf, wf = (x.float().cpu().numpy() for x in (q, k, w))
    ref = I.scores_ref(qf, kf, wf, ratio, q_offset)
    assert got.shape == (B, S, T) and got.dtype == np.float32
    masked = ~np.isfinite(ref)
    assert np.array_equal(~np.isfinite(got), masked), "group-causal -inf mask differs"
    fin = ~masked
    if fin.any():
        # reference criterion (dense_attn/ref.py:65): err <= 2 x torch-bf16 err + 1e-5; the
        # kernel's inputs are bf16 and it accumulates in fp32, so its error is fp32 noise
        err = np.abs(got[fin] - ref[fin]).max()
        scale = np.abs(ref[fin]).max()
        assert err <= 1e-5 * max(1.0, scale), f"max err {err}"


@pytest.mark.gpu
@pytest.mark.parametrize("heads", [4, 32, 64])
@pytest.mark.parametrize("dim", [64, 96, 128, 256])
def test_scores_match_reference(cuda, dim, heads):
    import torch
    _check_scores(torch, cuda, 2, 256, heads, dim, 128, 2)


@pytest.mark.gpu
@pytest.mark.parametrize("S", [253, 254, 255])
def test_scores_partial_token_blocks(cuda, S):
    """64 heads take four-token query blocks drained by four warpgroups, two tokens each:
    a last block of one to three tokens leaves a warpgroup with nothing but its release."""
    import torch
    _check_scores(torch, cuda, 2, S, 64, 128, 160, 2, q_offset=64)


@pytest.mark.gpu
@pytest.mark.parametrize("S", [1, 2, 3])
@pytest.mark.parametrize("heads,dim", [(64, 64), (64, 128), (32, 64)])
def test_scores_few_tokens(cuda, S, heads, dim):
    """Query blocks of one to three tokens (decode-like): tiles of at most 128 query columns
    run on four 128-column TMEM accumulators when the key ring has four stages, wider ones on
    two; the epilogue waits on each key stage's barrier either way."""
    import torch
    _check_scores(torch, cuda, 3, S, heads, dim, 700, 2, q_offset=600)


@pytest.mark.gpu
@pytest.mark.parametrize("ratio", [1, 2, 4])
def test_compress_ratios(cuda, ratio):
    import torch
    _check_scores(torch, cuda, 1, 256, 32, 128, 256 // ratio, ratio)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [128, 400, 7])
def test_kv_lengths(cuda, T):
    import torch
    _check_scores(torch, cuda, 1, 256, 32, 128, T, 2)


@pytest.mark.gpu
def test_ragged_seq_and_offset(cuda):
    """S not a multiple of the token block, absolute positions (q_offset)."""
    import torch
    _check_scores(torch, cuda, 2, 258, 32, 128, 300, 4, q_offset=1000)


@pytest.mark.gpu
def test_empty_kv(cuda):
    import torch
    from mzoo_b200 import indexer
    q, k, w = _bf16_inputs(torch, cuda, 1, 256, 32, 128, 0)
    assert indexer.fwd(q, k, w, compress_ratio=2).shape == (1, 256, 0)
    assert (indexer.attn(q, k, w, compress_ratio=2, topk=8) == -1).all()


@pytest.mark.gpu
@pytest.mark.parametrize("topk,T", [(64, 128), (135, 128), (16, 400), (40, 397)])
def test_topk_bf16_exact(cuda, topk, T):
    import torch
    from mzoo_b200 import indexer
    B, S, Hi, Di, ratio = 2, 256, 32, 128, 1
    q, k, w = _bf16_inputs(torch, cuda, B, S, Hi, Di, T, seed=3)
    got = indexer.attn(q, k, w, compress_ratio=ratio, topk=topk).cpu().numpy()
    qf, kf, wf = (x.float().cpu().numpy() for x in (q, k, w))
    canon = I.canonical_scores(qf, kf, wf, None, None, ratio, 0, scale=float(np.float32(Di**-0.5)), fp8=False)
    assert np.array_equal(got, I.canonical_topk(canon, topk, ratio))
    # and the same sets as the reference's fp32 scores + topk
    ref = I.topk_ref(I.scores_ref(qf, kf, wf, ratio), topk)
    assert np.array_equal(got, ref.astype(np.int32))


@pytest.mark.gpu
def test_topk_all_tied_rows(cuda):
    """Zero head weights make every visible score exactly 0: the selection must fall back
    to the lowest indices (the reference's tie rule), for rows shorter and longer than topk."""
    import torch
    from mzoo_b200 import indexer
    B, S, Hi, Di, T, ratio, topk = 1, 64, 32, 128, 300, 1, 16
    q, k, w = _bf16_inputs(torch, cuda, B, S, Hi, Di, T, seed=5)
    got = indexer.attn(q, k, torch.zeros_like(w), compress_ratio=ratio, topk=topk).cpu().numpy()
    for s in range(S):
        n = min(topk, s + 1)
        assert np.array_equal(got[0, s, :n], np.arange(n)) and (got[0, s, n:] == -1).all(), s


@pytest.mark.gpu
def test_topk_tied_block_exact(cuda):
    """300 zero key rows score exactly 0 for every query; with positive head weights every
    other key scores above 0 and the cut falls inside the tie: the selected bin holds more
    keys than are ranked directly (radix select), and the exact re-scoring of the band
    breaks the tie by the lower index."""
    import torch
    from mzoo_b200 import indexer
    B, S, Hi, Di, T, ratio, topk = 1, 64, 64, 128, 1200, 1, 1000
    q, k, w = _bf16_inputs(torch, cuda, B, S, Hi, Di, T, seed=9)
    w = w.abs()
    k[:, 500:800] = 0
    got = indexer.attn(q, k, w, compress_ratio=ratio, topk=topk, q_offset=T).cpu().numpy()
    qf, kf, wf = (x.float().cpu().numpy() for x in (q, k, w))
    canon = I.canonical_scores(qf, kf, wf, None, None, ratio, T, scale=float(np.float32(Di**-0.5)), fp8=False)
    pos = (canon[0] > 0).sum(axis=1)
    assert ((pos < topk) & (pos + 300 >= topk)).all(), "the cut should fall in the tie"
    assert np.array_equal(got, I.canonical_topk(canon, topk, ratio, T))


@pytest.mark.gpu
def test_topk_wide_band_exact(cuda):
    """A band 2^10 times wider than the error bound needs (eps passed to the op) spans many
    linear bins, so every key is scanned for it; exact re-scoring gives the same sets."""
    import torch
    from mzoo_b200 import indexer, ops
    B, S, Hi, Di, T, ratio, topk = 2, 128, 64, 128, 1024, 1, 64
    q8, sq, k8, sk, w = _fp8_case(torch, cuda, B, S, Hi, Di, T, 11)
    qp, kp, wp, sqp, skp, scale, dt = indexer._prep(q8, k8, w, (sq, sk), None)
    sc = indexer._scores(qp, kp, wp, sqp, skp, ratio, T, scale, dt, False, True)
    got = ops.indexer_topk(sc, qp, kp, wp, sqp, skp, None, None, ratio, T, scale, dt, topk, indexer.EPS * 1024,
                           indexer.KB_PARTS, True).cpu().numpy()
    qv, kv = q8.float().cpu().numpy(), k8.float().cpu().numpy()
    canon = I.canonical_scores(qv, kv, w.cpu().numpy(), sq.cpu().numpy(), sk.cpu().numpy(), ratio, T)
    assert np.array_equal(got, I.canonical_topk(canon, topk, ratio, T))


def _fp8_case(torch, dev, B, S, Hi, Di, T, seed):
    from mzoo_b200 import indexer
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, S, Hi, Di, generator=g)
    k = torch.randn(B, T, Di, generator=g)
    w = torch.randn(B, S, Hi, generator=g) / 8
    q8, sq = indexer.quantize_fp8(q.to(dev))
    k8, sk = indexer.quantize_fp8(k.to(dev))
    return q8, sq, k8, sk, w.to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("q_offset", [0, 1536])
def test_topk_fp8_exact(cuda, q_offset):
    """BASELINE config 2 at reduced size: fp8 q/k with absmax scales, ratio 4, top-k 64."""
    import torch
    from mzoo_b200 import indexer
    B, S, Hi, Di, T, ratio, topk = 2, 512, 64, 128, 512, 4, 64
    q8, sq, k8, sk, w = _fp8_case(torch, cuda, B, S, Hi, Di, T, 7)
    got = indexer.attn(q8, k8, w, compress_ratio=ratio, topk=topk, q_offset=q_offset, scales=(sq, sk))
    qv = q8.float().cpu().numpy()
    kv = k8.float().cpu().numpy()
    canon = I.canonical_scores(qv, kv, w.cpu().numpy(), sq.cpu().numpy(), sk.cpu().numpy(), ratio, q_offset)
    assert np.array_equal(got.cpu().numpy(), I.canonical_topk(canon, topk, ratio, q_offset))


@pytest.mark.gpu
@pytest.mark.parametrize("topk", [5, 12, 30])
def test_topk_fp8_matches_reference_fixture(cuda, topk):
    """The FP8 kernel path (e4m3 codes + scales, softmax_scale = Di**-0.5) on the reference
    fixture's own inputs selects the reference's index sets."""
    import torch
    from mzoo_b200 import indexer
    d = _golden_fp8()
    ratio = int(d["params"][0])
    di = d["q"].shape[-1]
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)  # noqa: E731
    q8, k8 = t(d["q_codes"]).view(torch.float8_e4m3fn), t(d["k_codes"]).view(torch.float8_e4m3fn)
    got = indexer.attn(q8, k8, t(d["w"]), compress_ratio=ratio, topk=topk, scales=(t(d["sq"]), t(d["sk"])),
                       softmax_scale=di**-0.5).cpu().numpy()
    r = np.sort(np.where(d[f"topk{topk}"] < 0, 1 << 30, d[f"topk{topk}"]), -1)
    assert np.array_equal(got, np.where(r == 1 << 30, -1, r).astype(np.int32))


def _to_pages(torch, k8, sk, T, seed, extra=5):
    """The keys [B, >=T, Di] (+ scales [B, >=T]) laid out as a pool of 64-key pages in random
    order, pages past each batch's keys holding junk -> (pool [P,64,Di], scales [P,64],
    page table [B, pages])."""
    B, _, Di = k8.shape
    pages = -(-T // 64)
    g = torch.Generator(device="cpu").manual_seed(seed)
    P = B * pages + extra
    perm = torch.randperm(P, generator=g)[:B * pages].view(B, pages)
    junk = torch.randint(0, 120, (P, 64, Di), generator=g, dtype=torch.uint8)
    pool = junk.to(k8.device).view(torch.float8_e4m3fn)
    spool = (torch.rand(P, 64, generator=g) + 0.5).to(k8.device)
    for b in range(B):
        for pg in range(pages):
            n = min(64, T - pg * 64)
            pool[perm[b, pg], :n] = k8[b, pg * 64:pg * 64 + n]
            spool[perm[b, pg], :n] = sk[b, pg * 64:pg * 64 + n]
    return pool, spool, perm.to(torch.int32).to(k8.device)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", ["decode", "prefill"])
def test_paged_keys_match_dense(cuda, shape):
    """Keys reached through a page table of 64-key pages (a paged decode cache) give the
    same scores bit for bit and the same index sets as the same keys stored dense."""
    import torch
    from mzoo_b200 import indexer
    if shape == "decode":
        B, S, Hi, Di, T, ratio, topk = 6, 1, 64, 128, 4000, 4, 256
        q8, sq, k8, sk, w = _fp8_case(torch, cuda, B, S, Hi, Di, T, 31)
        lens = torch.tensor([16000, 1000, 9001, 4097, 15999, 777], dtype=torch.int32)
        kw = dict(compress_ratio=ratio, scales=(sq, sk), q_pos=(lens - 1).view(B, 1).to(cuda))
    else:
        B, S, Hi, Di, T, ratio, topk = 2, 200, 64, 128, 300, 1, 64
        q8, sq, k8, sk, w = _fp8_case(torch, cuda, B, S, Hi, Di, T, 32)
        kw = dict(compress_ratio=ratio, scales=(sq, sk), q_offset=100)
    pool, spool, pt = _to_pages(torch, k8, sk, T, 7)
    kwp = dict(kw, scales=(sq, spool), k_page_table=pt)
    dense = indexer.attn(q8, k8, w, topk=topk, check=True, **kw)
    paged = indexer.attn(q8, pool, w, topk=topk, check=True, **kwp)
    assert torch.equal(dense, paged)
    sd = indexer.fwd(q8, k8, w, **kw)
    sp = indexer.fwd(q8, pool, w, **kwp)
    assert torch.equal(sd, sp[:, :, :T]) and torch.isneginf(sp[:, :, T:]).all()


@pytest.mark.gpu
def test_decode_shaped_topk_fp8_exact(cuda):
    """One query per sequence at its own position (paged decode, BASELINE config 4 at reduced
    size): per-batch q_pos, few (batch, block) items, so the score kernel splits key ranges."""
    import torch
    from mzoo_b200 import indexer
    B, Hi, Di, T, ratio, topk = 6, 64, 128, 4000, 4, 256
    q8, sq, k8, sk, w = _fp8_case(torch, cuda, B, 1, Hi, Di, T, 21)
    lens = torch.tensor([16000, 1000, 9001, 4097, 15999, 777], dtype=torch.int32)
    pos = (lens - 1).view(B, 1).to(cuda)
    got = indexer.attn(q8, k8, w, compress_ratio=ratio, topk=topk, scales=(sq, sk), q_pos=pos).cpu().numpy()
    sc = indexer.fwd(q8, k8, w, compress_ratio=ratio, scales=(sq, sk), q_pos=pos).cpu().numpy()
    qv, kv, wn, sqn, skn = (x.float().cpu().numpy() for x in (q8, k8, w, sq, sk))
    for b in range(B):
        canon = I.canonical_scores(qv[b:b + 1], kv[b:b + 1], wn[b:b + 1], sqn[b:b + 1], skn[b:b + 1], ratio,
                                   int(pos[b, 0]))
        assert np.array_equal(got[b:b + 1], I.canonical_topk(canon, topk, ratio, int(pos[b, 0]))), b
        vis = int(lens[b]) // ratio
        assert np.isneginf(sc[b, 0, vis:]).all() and np.isfinite(sc[b, 0, :vis]).all()
        rel = np.abs(sc[b, 0, :vis] - canon[0, 0, :vis]).max() / np.abs(canon[0, 0, :vis]).max()
        assert rel < 1e-5, (b, rel)


@pytest.mark.gpu
def test_fp8_score_error_within_bound(cuda):
    """The fp32 tensor-core scores stay well inside the bound the top-k relies on:
    |approx - exact| <= EPS * A_s * max_t B_t, with a 16x margin."""
    import torch
    from mzoo_b200 import indexer
    B, S, Hi, Di, T, ratio = 1, 512, 64, 128, 1024, 1
    q8, sq, k8, sk, w = _fp8_case(torch, cuda, B, S, Hi, Di, T, 11)
    approx = indexer.fwd(q8, k8, w, compress_ratio=ratio, q_offset=T, scales=(sq, sk)).cpu().numpy()
    qv, kv, wn, sqn, skn = (x.float().cpu().numpy() for x in (q8, k8, w, sq, sk))
    canon = I.canonical_scores(qv, kv, wn, sqn, skn, ratio, T)
    A, Bt = I.bound_factors(qv, kv, wn, sqn, skn)
    bound = A[..., None] * Bt.max(-1)[:, None, None]
    ratio_err = (np.abs(approx.astype(np.float64) - canon) / bound).max()
    print(f"max |approx-exact| / (A_s max B_t) = {ratio_err:.3e} (EPS = {indexer.EPS:.3e})")
    assert ratio_err <= indexer.EPS / 16


# ----------------------------------------------------------------------------- backward

def test_oracle_bwd_matches_reference_autograd():
    d = _golden()
    dq, dk, dw = I.scores_bwd_ref(d["q"], d["k"], d["w"], d["bwd.dl"], 2)
    np.testing.assert_allclose(dq, d["bwd.dq"], atol=2e-6)
    np.testing.assert_allclose(dk, d["bwd.dk"], atol=2e-6)
    np.testing.assert_allclose(dw, d["bwd.dw"], atol=5e-6)


def _grad_close(got, ref, what, rel=1e-2, atol=2e-2):
    got = got.float().cpu().numpy()
    err = np.abs(got - ref).max()
    scale = np.abs(ref).max()
    print(f"{what}: max err {err:.3e} (ref max {scale:.2e})")
    assert err <= atol + rel * scale, what


@pytest.mark.gpu
@pytest.mark.parametrize("heads,dim,ratio", [(4, 64, 2), (32, 128, 4), (64, 128, 1), (16, 128, 2), (8, 96, 2),
                                             (4, 256, 2), (32, 256, 2), (128, 256, 4)])
def test_bwd_matches_oracle(cuda, heads, dim, ratio):
    """indexer/bwd_test.py:29-62: dq / dk / dw against autograd through the fp32 scores."""
    import torch
    from mzoo_b200 import indexer
    B, S, T = 2, 256, 160
    q, k, w = _bf16_inputs(torch, cuda, B, S, heads, dim, T, seed=heads + dim)
    g = torch.Generator(device="cpu").manual_seed(5)
    dl = torch.randn(B, S, T, generator=g).to(cuda)
    dq, dk, dw = indexer.bwd(q, k, w, dl, compress_ratio=ratio)
    rq, rk, rw = I.scores_bwd_ref(q.float().cpu().numpy(), k.float().cpu().numpy(), w.cpu().numpy(),
                                  dl.cpu().numpy(), ratio)
    _grad_close(dq, rq, "dq")
    _grad_close(dk, rk, "dk")
    _grad_close(dw, rw, "dw", rel=1e-4, atol=1e-4)


@pytest.mark.gpu
def test_bwd_ignores_masked_junk(cuda):
    """indexer/bwd_test.py:86-108: NaN / huge values at masked positions change nothing."""
    import torch
    from mzoo_b200 import indexer
    B, S, T, ratio = 1, 256, 128, 2
    q, k, w = _bf16_inputs(torch, cuda, B, S, 32, 128, T, seed=1)
    dl = torch.randn(B, S, T, device=cuda)
    s_idx = torch.arange(S, device=cuda)[:, None]
    t_idx = torch.arange(T, device=cuda)[None, :]
    masked = t_idx >= (s_idx + 1) // ratio
    clean = indexer.bwd(q, k, w, dl.masked_fill(masked, 0.0), compress_ratio=ratio)
    junk = indexer.bwd(q, k, w, dl.masked_fill(masked, float("nan")), compress_ratio=ratio)
    for a_, b_ in zip(clean, junk):
        assert torch.equal(a_, b_)


@pytest.mark.gpu
def test_scores_autograd_and_fp4_ste(cuda):
    """indexer/attn.py:53 + bwd_test.py:147-190: feature-off forward equals fwd bit for bit;
    the fp4 STE forward equals fwd on quantised inputs and its gradient is the plain one."""
    import torch
    from mzoo_b200 import indexer, quant
    q, k, w = _bf16_inputs(torch, cuda, 1, 256, 32, 128, 128, seed=2)
    qg, kg, wg = (x.clone().requires_grad_() for x in (q, k, w))
    out = indexer.scores(qg, kg, wg, compress_ratio=2)
    assert torch.equal(out, indexer.fwd(q, k, w, compress_ratio=2))
    dl = torch.randn_like(out).masked_fill(torch.isinf(out), 0.0)
    out.backward(dl)
    dq, dk, dw = indexer.bwd(q, k, w, dl, compress_ratio=2)
    assert torch.equal(qg.grad, dq) and torch.equal(kg.grad, dk) and torch.equal(wg.grad, dw)
    qg2, kg2 = q.clone().requires_grad_(), k.clone().requires_grad_()
    out2 = indexer.scores(qg2, kg2, w, compress_ratio=2, fake_quant_fp4=True)
    ref2 = indexer.fwd(quant._fake_quant_fp4_block(q, 32), quant._fake_quant_fp4_block(k, 32), w, compress_ratio=2)
    assert torch.equal(out2, ref2)
    out2.backward(dl)
    dq2, dk2, _ = indexer.bwd(quant._fake_quant_fp4_block(q, 32), quant._fake_quant_fp4_block(k, 32), w, dl,
                              compress_ratio=2)
    assert torch.equal(qg2.grad, dq2) and torch.equal(kg2.grad, dk2)
