"""Two-level indexer selection: the oracle pinned to the reference's own outputs (CPU), the
sm_100a kernels against the oracle and the golden vectors (GPU).

Reference behaviour mirrored (``select_candidate_blocks``, archs/dsv4/modeling_deepseek_v41.py
:427-454; level two :566-578) and the cases its plan asks for
(tickets/0009-indexer-hierarchical.md "Acceptance"): T not a multiple of the block size,
fewer reachable blocks than topk_blocks, a query whose newest block is also its best block,
the pinned partial block and the drop of -inf picks.  Ties go to the lower index here; the
golden inputs are continuous random values, so they hold none.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import candidates as C


def _golden():
    return np.load(os.path.join(GOLDEN, "candidates.npz"))


def _cases(d):
    n = len([k for k in d.files if k.endswith(".params")])
    for c in range(n):
        key = f"c{c}."
        yield {k[len(key):]: d[k] for k in d.files if k.startswith(key)}


# ----------------------------------------------------------------------------- CPU: oracle pin

def test_oracle_level_one_matches_reference_golden():
    for case in _cases(_golden()):
        bs, tb, _ = (int(x) for x in case["params"])
        got = C.candidate_mask_ref(case["logits"], case["clen"], tb, bs)
        assert np.array_equal(got, case["mask"])


def test_oracle_level_two_matches_reference_golden():
    for case in _cases(_golden()):
        _, _, topk = (int(x) for x in case["params"])
        got = C.candidate_topk_ref(case["scores2"], case["mask"], topk)
        assert np.array_equal(got, case["topk_idx"])


def test_oracle_pins_newest_block_and_drops_unreachable():
    # one row, 3 reachable positions in block 0 of 4-wide blocks; block 0 pinned even though
    # a later block (unreachable in the reference's sense only by its -inf scores) is empty
    logits = np.array([[0.5, -3.0, -2.0, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf]], np.float32)
    assert np.array_equal(C.candidate_blocks_ref(logits, np.array([3]), 2, 4), [[0, -1]])
    # compress_len 0: nothing pinned, nothing reachable
    assert np.array_equal(C.candidate_blocks_ref(np.full((1, 9), -np.inf, np.float32), np.array([0]), 2, 4),
                          [[-1, -1]])
    # the pinned block wins over a better full block when only one is kept
    logits = np.array([[9.0, 9.0, 1.0, 0.0, 0.0]], np.float32)
    assert np.array_equal(C.candidate_blocks_ref(logits, np.array([5]), 1, 2), [[2]])


def test_oracle_tie_rule_brute_force():
    """The reference's fixtures hold no ties; check the oracle's lower-index rule against a
    plain-Python restatement on coarse (tie-heavy) rows, with -inf and pinned blocks."""
    rng = np.random.default_rng(21)
    for _ in range(60):
        T, bs = int(rng.integers(1, 60)), int(rng.integers(1, 6))
        tb, topk = int(rng.integers(1, 8)), int(rng.integers(1, 12))
        clen = int(rng.integers(0, T + 3))
        row = np.round(rng.standard_normal(T) * 2) / 2
        row[np.arange(T) >= clen] = -np.inf
        logits = row.astype(np.float32)[None]
        nb = -(-T // bs)
        score = [max([float(logits[0, t]) for t in range(b * bs, min(T, b * bs + bs))]) for b in range(nb)]
        last = (clen - 1) // bs
        if 0 <= last < nb:
            score[last] = float("inf")
        order = sorted(range(nb), key=lambda b: (-score[b], b))[:min(tb, nb)]
        picks = sorted(b for b in order if score[b] > float("-inf"))
        want = picks + [-1] * (tb - len(picks))
        assert C.candidate_blocks_ref(logits, np.array([clen]), tb, bs).tolist() == [want]
        mask = C.candidate_mask_ref(logits, np.array([clen]), tb, bs)
        s2 = (np.round(rng.standard_normal(T) * 2) / 2).astype(np.float32)[None]
        vals = [float(s2[0, t]) if mask[0, t] else float("-inf") for t in range(T)]
        order = sorted(range(T), key=lambda t: (-vals[t], t))[:min(topk, T)]
        picks = sorted(t for t in order if vals[t] > float("-inf"))
        want = picks + [-1] * (min(topk, T) - len(picks))
        assert C.candidate_topk_ref(s2, mask, topk).tolist() == [want]


# ----------------------------------------------------------------------------- GPU: kernels

def _rand_case(rng, rows, T, ratio, off, ties=False):
    pos = off + np.arange(rows) * max(1, (T * ratio) // max(rows, 1))
    clen = (pos + 1) // ratio
    vals = rng.standard_normal((rows, T)).astype(np.float32)
    if ties:  # coarse values: many equal block maxima and equal scores
        vals = np.round(vals * 2) / 2
    logits = np.where(np.arange(T)[None, :] < clen[:, None], vals, -np.inf).astype(np.float32)
    return logits, clen.astype(np.int64)


@pytest.mark.gpu
def test_kernels_match_reference_golden(cuda):
    import torch
    from mzoo_b200 import candidates as K
    for case in _cases(_golden()):
        bs, tb, topk = (int(x) for x in case["params"])
        lg = torch.from_numpy(case["logits"]).to(cuda)
        cl = torch.from_numpy(case["clen"]).to(cuda).unsqueeze(-1)
        mask = K.select_candidate_blocks(lg, cl, tb, bs)
        assert np.array_equal(mask.cpu().numpy(), case["mask"])
        sc = torch.from_numpy(case["scores2"]).to(cuda)
        got = K.candidate_topk(sc, mask, topk)
        assert np.array_equal(got.cpu().numpy(), case["topk_idx"])
        blocks = K.candidate_blocks(lg, cl, tb, bs)
        got = K.candidate_topk(sc, blocks, topk, block_size=bs)
        assert np.array_equal(got.cpu().numpy(), case["topk_idx"])


@pytest.mark.gpu
@pytest.mark.parametrize("rows,T,ratio,bs,tb,topk,off,ties", [
    (64, 4096, 4, 8, 64, 512, 12288, False),   # C2-like row length, selection active
    (32, 16384, 1, 8, 2048, 512, 0, False),    # the model's defaults: 2048 blocks of 8
    (16, 20000, 1, 8, 2048, 512, 4000, False),  # 2500 blocks: T not a multiple of 8
    (32, 1000, 1, 8, 40, 100, 0, True),        # many tied block maxima and scores
    (8, 131072, 1, 8, 2048, 512, 100000, False),  # the 16384-block maximum
    (5, 3, 1, 8, 4, 2, 0, False),              # tiny rows, one partial block
])
def test_kernels_match_oracle(cuda, rows, T, ratio, bs, tb, topk, off, ties):
    import torch
    from mzoo_b200 import candidates as K
    rng = np.random.default_rng(rows * 7 + T)
    logits, clen = _rand_case(rng, rows, T, ratio, off, ties)
    lg = torch.from_numpy(logits).to(cuda)
    cl = torch.from_numpy(clen).to(cuda)
    blocks = K.candidate_blocks(lg, cl, tb, bs).cpu().numpy()
    ref_blocks = C.candidate_blocks_ref(logits, clen, tb, bs)
    assert np.array_equal(blocks, ref_blocks)
    mask = K.select_candidate_blocks(lg, cl, tb, bs).cpu().numpy()
    ref_mask = C.candidate_mask_ref(logits, clen, tb, bs)
    assert np.array_equal(mask, ref_mask)
    scores2, _ = _rand_case(rng, rows, T, ratio, off, ties)
    sc = torch.from_numpy(scores2).to(cuda)
    ref = C.candidate_topk_ref(scores2, ref_mask, topk)
    got = K.candidate_topk(sc, torch.from_numpy(blocks).to(cuda), topk, block_size=bs).cpu().numpy()
    assert np.array_equal(got, ref)
    got = K.candidate_topk(sc, torch.from_numpy(mask).to(cuda), topk).cpu().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.gpu
def test_kernels_nan_and_empty(cuda):
    import torch
    from mzoo_b200 import candidates as K
    logits = np.array([[np.nan, 1.0, -np.inf, 2.0], [np.nan, np.nan, np.nan, np.nan]], np.float32)
    clen = np.array([4, 0])
    lg, cl = torch.from_numpy(logits).to(cuda), torch.from_numpy(clen).to(cuda)
    got = K.candidate_blocks(lg, cl, 1, 2).cpu().numpy()
    assert np.array_equal(got, C.candidate_blocks_ref(logits, clen, 1, 2))
    got = K.candidate_topk(lg, torch.ones(2, 4, dtype=torch.bool, device=cuda), 3).cpu().numpy()
    assert np.array_equal(got, C.candidate_topk_ref(logits, np.ones((2, 4), bool), 3))
    # zero rows and zero width
    e = K.candidate_blocks(torch.empty(0, 16, device=cuda), torch.empty(0, dtype=torch.int64, device=cuda), 4, 8)
    assert e.shape == (0, 4)
    assert K.candidate_topk(torch.empty(3, 0, device=cuda), torch.empty(3, 0, dtype=torch.bool, device=cuda),
                            5).shape == (3, 0)


@pytest.mark.gpu
def test_kernels_reject_too_many_blocks(cuda):
    import torch
    from mzoo_b200 import candidates as K
    lg = torch.zeros(1, 16384 * 8 + 1, device=cuda)
    with pytest.raises(AssertionError, match="blocks per row"):
        K.candidate_blocks(lg, torch.ones(1, dtype=torch.int64, device=cuda), 8, 8)


@pytest.mark.gpu
def test_kernels_unaligned_rows(cuda):
    """A logits view 4 bytes past an aligned address takes the scalar block-max path."""
    import torch
    from mzoo_b200 import candidates as K
    rng = np.random.default_rng(11)
    logits, clen = _rand_case(rng, 12, 4096, 1, 3000)
    flat = torch.zeros(logits.size + 1, device=cuda)
    flat[1:] = torch.from_numpy(logits.reshape(-1)).to(cuda)
    lg = flat[1:].view(12, 4096)
    assert lg.data_ptr() % 16 == 4
    got = K.candidate_blocks(lg, torch.from_numpy(clen).to(cuda), 64, 8).cpu().numpy()
    assert np.array_equal(got, C.candidate_blocks_ref(logits, clen, 64, 8))


@pytest.mark.gpu
def test_level_two_streaming_path(cuda):
    """More listed blocks than the gathered kernel holds (5000 > 4096): the streaming kernel."""
    import torch
    from mzoo_b200 import candidates as K
    rng = np.random.default_rng(12)
    rows, T, bs, tb, topk = 6, 50000, 8, 5000, 300
    logits, clen = _rand_case(rng, rows, T, 1, 40000)
    blocks = C.candidate_blocks_ref(logits, clen, tb, bs)
    mask = C.candidate_mask_ref(logits, clen, tb, bs)
    scores2, _ = _rand_case(rng, rows, T, 1, 40000)
    got = K.candidate_topk(torch.from_numpy(scores2).to(cuda), torch.from_numpy(blocks).to(cuda), topk,
                           block_size=bs).cpu().numpy()
    assert np.array_equal(got, C.candidate_topk_ref(scores2, mask, topk))
