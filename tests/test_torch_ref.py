"""The torch float32 restatement of the reference's CPU path (``oracle/torch_ref.py``, the
arithmetic ``bench.py``'s reference arm times) pinned against the fixtures generated from
the reference itself, and against the numpy oracle for the two config-5 quant rules."""

import os

import numpy as np
import torch

from conftest import GOLDEN
from oracle import quant as Q
from oracle import torch_ref as R
from oracle.quant import bf16_to_f32


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_window_attention_matches_reference():
    d = _load("attention.npz")
    q, kv = torch.from_numpy(d["q"]), torch.from_numpy(d["kv"])
    for w in (1, 16, 40, 200):
        o, lse = R.window_attention(q, kv, w)
        np.testing.assert_allclose(o.numpy(), d[f"window{w}.o"], rtol=0, atol=1e-5)
        np.testing.assert_allclose(lse.numpy(), d[f"window{w}.lse"], rtol=0, atol=1e-5)


def test_indexer_scores_and_topk_match_reference():
    d = _load("indexer.npz")
    q, k, w = (torch.from_numpy(d[x]) for x in ("q", "k", "w"))
    sc = R.indexer_scores(q, k, w, 2, chunk=7)
    ref = d["scores"]
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(sc.numpy()), fin)
    np.testing.assert_allclose(sc.numpy()[fin], ref[fin], rtol=0, atol=1e-5)
    for topk in (4, 16, 25):
        got = np.sort(np.where(R.topk_indices(torch.from_numpy(ref), topk).numpy() < 0, 1 << 30,
                               R.topk_indices(torch.from_numpy(ref), topk).numpy()), -1)
        exp = np.sort(np.where(d[f"topk{topk}"] < 0, 1 << 30, d[f"topk{topk}"]), -1)
        assert np.array_equal(got, exp)


def test_pack_rows_matches_reference_fixture():
    d = _load("mla.npz")
    assert np.array_equal(R.pack_rows(torch.from_numpy(d["pre.kv"])).numpy(), d["pre.raw_rows"])
    assert np.array_equal(R.pack_rows(torch.from_numpy(d["pre.cmp"])).numpy(), d["pre.cmp_rows"])


def test_gathered_attention_matches_reference_prefill():
    d = _load("mla.npz")
    q_offset, window = (int(x) for x in d["pre.params"])
    raw = R.unpack_rows(torch.from_numpy(d["pre.raw_rows"]))
    cmp = R.unpack_rows(torch.from_numpy(d["pre.cmp_rows"]))
    q = torch.from_numpy(bf16_to_f32(d["pre.q"]))
    S, G = q.shape[0], cmp.shape[0]
    rows, counts = [], []
    for s in range(S):
        pos = s + q_offset
        sel = [int(i) for i in d["pre.idx"][s] if 0 <= i < G]
        rows.append(torch.cat([raw[max(0, pos - window + 1):pos + 1], cmp[sel]]))
        counts.append(rows[-1].shape[0])
    keys = torch.zeros(S, max(counts), 576)
    for s, r in enumerate(rows):
        keys[s, :r.shape[0]] = r
    o, lse = R.gathered_attention(q, keys, torch.tensor(counts), 576 ** -0.5)
    np.testing.assert_allclose(o.numpy(), d["pre.o"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(lse.numpy().T, d["pre.lse"], rtol=0, atol=2e-5)


def test_config5_quant_rules_match_numpy_oracle():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 256, generator=g) * torch.logspace(-3, 3, 256).view(1, 256)
    x[0, :32] = 0.0
    x[1, :32] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 4)
    got4 = R.fake_quant_fp4_ocp(x, 32).numpy()
    assert np.array_equal(got4, Q.fake_quant_fp4(x.numpy(), 32, "ocp"))
    got8 = R.fake_quant_fp8_absmax(x, 128).numpy()
    assert np.array_equal(got8, Q.fake_quant_fp8(x.numpy(), 128, "absmax"))
