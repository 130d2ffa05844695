"""swa_attn / csa2_attn (K == V shared-latent MQA, D <= 256): oracle pinned to the
reference's golden vectors (CPU); the sm_100a forward against the oracle (GPU).

Reference tests mirrored: ``swa_attn/fwd_test.py:53-130`` (window not tile-aligned,
window >= S, sinks), ``csa2_attn/fwd_test.py:82-195`` (topk > visible, non-power-of-2 G,
-1 padding, feature-off equals swa bit-for-bit).  Tolerance: the north-star max-abs
2e-2 + rel 1e-2 against the fp64 oracle on the same bf16 inputs.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import attention as A

ATOL, RTOL = 2e-2, 1e-2


def _golden():
    return np.load(os.path.join(GOLDEN, "attention.npz"))


# ----------------------------------------------------------------------------- CPU: oracle pin

@pytest.mark.parametrize("w", [1, 16, 40, 200])
def test_oracle_window_matches_reference(w):
    d = _golden()
    o, lse = A.attend(d["q"], d["kv"], window=w)
    np.testing.assert_allclose(o, d[f"window{w}.o"], atol=2e-6)
    np.testing.assert_allclose(lse, d[f"window{w}.lse"], atol=2e-6)


def test_oracle_sink_and_sparse_match_reference():
    d = _golden()
    o, lse = A.attend(d["q"], d["kv"], window=16, sinks=d["sinks"])
    np.testing.assert_allclose(o, d["window16sink.o"], atol=2e-6)
    np.testing.assert_allclose(lse, d["window16sink.lse"], atol=2e-6)
    o, lse = A.attend(d["q"], d["kv"], window=16, main_kv=d["main"], indices=d["idx"])
    np.testing.assert_allclose(o, d["sparse.o"], atol=2e-6)
    np.testing.assert_allclose(lse, d["sparse.lse"], atol=2e-6)


def test_oracle_gradients_match_reference_autograd():
    d = _golden()
    g = A.attend_bwd(d["q"], d["kv"], d["bwd.do"], window=16, sinks=d["sinks"])
    np.testing.assert_allclose(g["dq"], d["bwd.dq"], atol=5e-6)
    np.testing.assert_allclose(g["dkv"], d["bwd.dkv"].reshape(g["dkv"].shape), atol=5e-6)
    np.testing.assert_allclose(g["dsinks"], d["bwd.dsinks"], atol=5e-6)


# ----------------------------------------------------------------------------- GPU

def _inputs(torch, dev, B, S, H, D, G=0, topk=0, ratio=4, seed=0, dup=False, holes=False, sinks=False, sep_v=False):
    rng = np.random.default_rng(seed)
    f = lambda *s: torch.from_numpy(rng.standard_normal(s).astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    q, kv = f(B, S, H, D), f(B, S, 1, D)
    v = f(B, S, 1, D) if sep_v else None
    main = f(B, G, 1, D) if G else None
    idx = None
    if topk:
        idx = np.full((B, S, topk), -1, np.int32)
        for b in range(B):
            for s in range(S):
                vis = min(G, (s + 1) // ratio)
                sel = np.sort(rng.permutation(vis)[:topk]) if vis else []
                idx[b, s, :len(sel)] = sel
                if dup and len(sel) >= 2:
                    idx[b, s, 1] = idx[b, s, 0]
                if holes and len(sel) >= 3:
                    idx[b, s, 2] = -1
        idx = torch.from_numpy(idx)
    sk = torch.from_numpy(rng.standard_normal(H).astype(np.float32)) if sinks else None
    mv = lambda t: None if t is None else t.to(dev)  # noqa: E731
    return mv(q), mv(kv), mv(v), mv(main), mv(idx), mv(sk)


def _np(t):
    return None if t is None else t.float().cpu().numpy()


def _check(o, lse, ref_o, ref_lse, what):
    o, lse = _np(o), _np(lse)
    eo = np.abs(o - ref_o).max()
    el = np.abs(lse - ref_lse).max()
    print(f"{what}: max|o-ref|={eo:.3e} max|lse-ref|={el:.3e}")
    assert np.all(np.abs(o - ref_o) <= ATOL + RTOL * np.abs(ref_o)), f"{what}: o err {eo}"
    assert np.all(np.abs(lse - ref_lse) <= ATOL + RTOL * np.abs(ref_lse)), f"{what}: lse err {el}"


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 96, 128, 256])
@pytest.mark.parametrize("H", [4, 16, 64])
def test_swa_fwd(cuda, D, H):
    import torch
    from mzoo_b200 import swa_attn
    q, kv, _, _, _, _ = _inputs(torch, cuda, 2, 160, H, D, seed=D + H)
    o, lse = swa_attn.fwd(q, kv, window=100)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=100)
    _check(o, lse, ref_o, ref_lse, f"swa D{D} H{H}")


@pytest.mark.gpu
def test_swa_fwd_config1_shape(cuda):
    """BASELINE config 1 (the reference's CPU case): B1, S=2048, 16 heads sharing one KV
    head, D=128, window 128, scale 1/sqrt(128) -- on the bf16 kernel vs the fp64 oracle."""
    import torch
    from mzoo_b200 import swa_attn
    q, kv, _, _, _, _ = _inputs(torch, cuda, 1, 2048, 16, 128, seed=1)
    o, lse = swa_attn.fwd(q, kv, window=128)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=128)
    _check(o, lse, ref_o, ref_lse, "swa config 1")


@pytest.mark.gpu
@pytest.mark.parametrize("window", [1, 128, 513, 4096])
def test_swa_windows_and_sinks(cuda, window):
    import torch
    from mzoo_b200 import swa_attn
    q, kv, _, _, _, sk = _inputs(torch, cuda, 1, 600, 32, 128, seed=window, sinks=True)
    o, lse = swa_attn.fwd(q, kv, window=window, sinks=sk)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=window, sinks=_np(sk))
    _check(o, lse, ref_o, ref_lse, f"swa window {window}")


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,D,window", [(2, 300, 64, 128, 160), (1, 1200, 64, 128, 512), (2, 700, 16, 64, 300),
                                            (1, 500, 8, 256, 200)])
def test_swa_separate_v(cuda, B, S, H, D, window):
    # several query-tile items per CTA (S = 1200 at 64 heads is 600 items), ragged last
    # tiles, head dims 64 / 128 (two softmax warpgroups) and 256
    import torch
    from mzoo_b200 import swa_attn
    q, kv, v, _, _, _ = _inputs(torch, cuda, B, S, H, D, seed=4, sep_v=True)
    o, lse = swa_attn.fwd(q, kv, window=window, v=v)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=window, v=_np(v)[:, :, 0])
    _check(o, lse, ref_o, ref_lse, f"swa K!=V S{S} H{H} D{D}")


@pytest.mark.gpu
@pytest.mark.parametrize("H,D,G,topk", [(64, 128, 100, 100), (16, 64, 37, 48), (64, 256, 70, 64), (4, 128, 50, 135),
                                         (16, 96, 40, 32)])
def test_csa2_fwd(cuda, H, D, G, topk):
    import torch
    from mzoo_b200 import csa2_attn
    q, kv, _, main, idx, sk = _inputs(torch, cuda, 2, 200, H, D, G=G, topk=topk, seed=G + topk, holes=True,
                                      sinks=True)
    o, lse = csa2_attn.fwd(q, kv, main, idx, window=100, compress_ratio=4, sinks=sk)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=100, main_kv=_np(main)[:, :, 0],
                              indices=idx.cpu().numpy(), sinks=_np(sk))
    _check(o, lse, ref_o, ref_lse, f"csa2 H{H} D{D} G{G} topk{topk}")


@pytest.mark.gpu
def test_csa2_duplicates_count_twice(cuda):
    import torch
    from mzoo_b200 import csa2_attn
    q, kv, _, main, idx, _ = _inputs(torch, cuda, 1, 128, 64, 128, G=40, topk=32, seed=8, dup=True)
    o, lse = csa2_attn.fwd(q, kv, main, idx, window=64, compress_ratio=4)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=64, main_kv=_np(main)[:, :, 0],
                              indices=idx.cpu().numpy())
    _check(o, lse, ref_o, ref_lse, "csa2 duplicates")


@pytest.mark.gpu
def test_csa2_feature_off_equals_swa_bitwise(cuda):
    """csa2_attn/fwd_test.py:145-168: all -1 indices, or G == 0, is swa_attn bit for bit."""
    import torch
    from mzoo_b200 import csa2_attn, swa_attn
    q, kv, _, main, idx, sk = _inputs(torch, cuda, 2, 256, 64, 128, G=64, topk=64, seed=2, sinks=True)
    ref = swa_attn.fwd(q, kv, window=128, sinks=sk)
    got = csa2_attn.fwd(q, kv, main, torch.full_like(idx, -1), window=128, compress_ratio=4, sinks=sk)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    empty = main[:, :0]
    got = csa2_attn.fwd(q, kv, empty, idx, window=128, compress_ratio=4, sinks=sk)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])


# ----------------------------------------------------------------------------- GPU: backward

def _check_grad(got, ref, what, torch_bf16=None):
    """Gradients: max-abs error within 2e-2 + 1e-2 * max|ref| (taken
    relative to the tensor's scale: a bf16 backward rounds P and dS to 8 bits, so keys fed by
    near-one probabilities carry errors near 1e-2 of the tensor maximum), and -- the reference's
    own acceptance criterion, ``dense_attn/ref.py:65`` -- at most 2x torch-bf16's error."""
    got = _np(got)
    err = np.abs(got - ref).max()
    scale = np.abs(ref).max()
    msg = f"{what}: max|d-ref|={err:.3e} (ref max {scale:.2e})"
    if torch_bf16 is not None:
        terr = np.abs(_np(torch_bf16) - ref).max()
        msg += f" torch-bf16 err {terr:.3e} ratio {err / max(terr, 1e-30):.2f}"
        assert err <= 2.0 * terr + 1e-5, msg
    print(msg)
    assert err <= ATOL + RTOL * scale, msg


def _torch_bf16_grads(torch, q, kv, do, window, sinks=None, v=None):
    """golden(dtype=bf16)-style reference: bf16 matmuls, fp32 softmax, bf16 probabilities,
    autograd for dq / dk / dv (golden_ref.py:83-100 with mm_dtype = bf16)."""
    B, S, H, D = q.shape
    qq = q.detach().clone().requires_grad_()
    kk = kv.detach().clone().requires_grad_()
    vv = (v if v is not None else kv).detach().clone().requires_grad_()
    qt = qq.transpose(1, 2)
    kt = kk.transpose(1, 2)
    vt = vv.transpose(1, 2)
    logits = torch.matmul(qt, kt.transpose(-1, -2)).float() * D**-0.5
    i = torch.arange(S, device=q.device)
    vis = (i[None, :] <= i[:, None]) & (i[None, :] > i[:, None] - window)
    logits = logits.masked_fill(~vis, float("-inf"))
    if sinks is not None:
        logits = torch.cat([logits, sinks.float().view(1, H, 1, 1).expand(B, H, S, 1)], -1)
    probs = torch.softmax(logits, -1)
    if sinks is not None:
        probs = probs[..., :-1]
    o = torch.matmul(probs.to(torch.bfloat16), vt).transpose(1, 2)
    o.backward(do)
    if v is None:  # K == V: the latent's gradient is dK + dV
        return qq.grad, (kk.grad.float() + vv.grad.float()), None
    return qq.grad, kk.grad, vv.grad


def _do(torch, dev, shape, seed):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(torch.bfloat16).to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("H,D,window", [(64, 128, 100), (16, 64, 37), (4, 128, 300), (16, 96, 100), (4, 256, 100),
                                        (16, 256, 37), (64, 256, 300)])
def test_swa_bwd(cuda, H, D, window):
    import torch
    from mzoo_b200 import swa_attn
    q, kv, _, _, _, sk = _inputs(torch, cuda, 2, 200, H, D, seed=H + D, sinks=True)
    o, lse = swa_attn.fwd(q, kv, window=window, sinks=sk)
    do = _do(torch, cuda, q.shape, 7)
    dq, dkv, dsinks = swa_attn.bwd(q, kv, o, lse, do, window=window, sinks=sk)
    ref = A.attend_bwd(_np(q), _np(kv)[:, :, 0], _np(do), window=window, sinks=_np(sk))
    tq, tk, _ = _torch_bf16_grads(torch, q, kv, do, window, sinks=sk)
    _check_grad(dq, ref["dq"], f"swa dq H{H} D{D}", tq)
    _check_grad(dkv[:, :, 0], ref["dkv"], f"swa dkv H{H} D{D}", tk[:, :, 0])
    _check_grad(dsinks, ref["dsinks"], f"swa dsinks H{H} D{D}")


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,H,D,window", [(2, 256, 64, 128, 200), (1, 1200, 64, 128, 512), (2, 700, 16, 64, 300)])
def test_swa_bwd_separate_v(cuda, B, S, H, D, window):
    # the window-only (separate V) kernels: several query-tile items per CTA (S = 1200 at 64
    # heads is 600 items), ragged last tiles, and head dim 64
    import torch
    from mzoo_b200 import swa_attn
    q, kv, v, _, _, _ = _inputs(torch, cuda, B, S, H, D, seed=11, sep_v=True)
    o, lse = swa_attn.fwd(q, kv, window=window, v=v)
    do = _do(torch, cuda, q.shape, 8)
    dq, dk, _, dv = swa_attn.bwd(q, kv, o, lse, do, window=window, v=v)
    ref = A.attend_bwd(_np(q), _np(kv)[:, :, 0], _np(do), window=window, v=_np(v)[:, :, 0])
    tq, tk, tv = _torch_bf16_grads(torch, q, kv, do, window, v=v)
    _check_grad(dq, ref["dq"], f"swa K!=V dq S{S} H{H} D{D}", tq)
    _check_grad(dk[:, :, 0], ref["dk"], f"swa K!=V dk S{S} H{H} D{D}", tk[:, :, 0])
    _check_grad(dv[:, :, 0], ref["dv"], f"swa K!=V dv S{S} H{H} D{D}", tv[:, :, 0])


@pytest.mark.gpu
@pytest.mark.parametrize("H,D,G,topk", [(64, 128, 100, 100), (16, 64, 37, 48), (16, 96, 40, 32), (4, 256, 40, 64),
                                        (16, 256, 100, 100), (64, 256, 70, 135)])
def test_csa2_bwd(cuda, H, D, G, topk):
    import torch
    from mzoo_b200 import csa2_attn
    q, kv, _, main, idx, sk = _inputs(torch, cuda, 2, 160, H, D, G=G, topk=topk, seed=G, dup=True, holes=True,
                                      sinks=True)
    o, lse = csa2_attn.fwd(q, kv, main, idx, window=64, compress_ratio=4, sinks=sk)
    do = _do(torch, cuda, q.shape, 9)
    dq, dkv, dmain, dsinks = csa2_attn.bwd(q, kv, main, idx, o, lse, do, window=64, compress_ratio=4, sinks=sk)
    ref = A.attend_bwd(_np(q), _np(kv)[:, :, 0], _np(do), window=64, main_kv=_np(main)[:, :, 0],
                       indices=idx.cpu().numpy(), sinks=_np(sk))
    _check_grad(dq, ref["dq"], f"csa2 dq H{H}")
    _check_grad(dkv[:, :, 0], ref["dkv"], f"csa2 dkv H{H}")
    _check_grad(dmain[:, :, 0], ref["dmain"], f"csa2 dmain H{H}")
    _check_grad(dsinks, ref["dsinks"], f"csa2 dsinks H{H}")


@pytest.mark.gpu
def test_swa_attn_autograd(cuda):
    """swa_attn/attn_test.py: gradients through the autograd wrapper."""
    import torch
    from mzoo_b200 import swa_attn
    q, kv, _, _, _, _ = _inputs(torch, cuda, 1, 130, 32, 128, seed=12)
    q.requires_grad_()
    kv.requires_grad_()
    do = _do(torch, cuda, q.shape, 10)
    swa_attn.attn(q, kv, window=50).backward(do)
    ref = A.attend_bwd(_np(q.detach()), _np(kv.detach())[:, :, 0], _np(do), window=50)
    _check_grad(q.grad, ref["dq"], "autograd dq")
    _check_grad(kv.grad[:, :, 0], ref["dkv"], "autograd dkv")


@pytest.mark.gpu
@pytest.mark.parametrize("sinks", [False, True])
def test_csa2_attn_autograd(cuda, sinks):
    """csa2_attn/attn_test.py:98-152 through the autograd wrapper (``csa2_attn/attn.py:20-55``):
    q, kv, main_kv (and sinks) receive the gradients ``csa2_attn.bwd`` gives, which match the
    oracle's closed form; duplicate and -1 indices; indices get no gradient."""
    import torch
    from mzoo_b200 import csa2_attn
    q, kv, _, main, idx, sk = _inputs(torch, cuda, 2, 160, 16, 128, G=48, topk=40, seed=21, dup=True, holes=True,
                                      sinks=sinks)
    do = _do(torch, cuda, q.shape, 13)
    leaves = [x.detach().clone().requires_grad_() for x in (q, kv, main)]
    sl = sk.detach().clone().requires_grad_() if sinks else None
    o = csa2_attn.attn(*leaves, idx, window=64, compress_ratio=4, sinks=sl)
    o.backward(do)
    o_ref, lse = csa2_attn.fwd(q, kv, main, idx, window=64, compress_ratio=4, sinks=sk)
    assert torch.equal(o.detach(), o_ref)
    dq, dkv, dmain, dsinks = csa2_attn.bwd(q, kv, main, idx, o_ref, lse, do, window=64, compress_ratio=4, sinks=sk)
    assert torch.equal(leaves[0].grad, dq) and torch.equal(leaves[1].grad, dkv)
    # dmain is accumulated by fp32 atomics (order varies run to run): compare to rounding
    assert (leaves[2].grad.float() - dmain.float()).abs().max() <= 2e-2
    ref = A.attend_bwd(_np(q), _np(kv)[:, :, 0], _np(do), window=64, main_kv=_np(main)[:, :, 0],
                       indices=idx.cpu().numpy(), sinks=_np(sk) if sinks else None)
    _check_grad(leaves[0].grad, ref["dq"], "autograd csa2 dq")
    _check_grad(leaves[1].grad[:, :, 0], ref["dkv"], "autograd csa2 dkv")
    _check_grad(leaves[2].grad[:, :, 0], ref["dmain"], "autograd csa2 dmain")
    if sinks:
        assert torch.equal(sl.grad, dsinks)
        _check_grad(sl.grad, ref["dsinks"], "autograd csa2 dsinks")


def test_head_groups():
    """csa2 launches for any head count (csa2_attn/fwd.py:65-67 accepts any H): H | 128 runs
    as is, H < 128 is padded to the next power of two, H > 128 runs in 128-head groups."""
    from mzoo_b200._attn_common import head_groups
    assert head_groups(64) == (64, 1) and head_groups(128) == (128, 1) and head_groups(1) == (1, 1)
    assert head_groups(48) == (64, 1) and head_groups(96) == (128, 1) and head_groups(6) == (8, 1)
    assert head_groups(256) == (128, 2) and head_groups(200) == (128, 2) and head_groups(384) == (128, 3)


@pytest.mark.gpu
@pytest.mark.parametrize("H", [6, 48, 96, 200, 256])
def test_csa2_any_heads(cuda, H):
    """Head counts that do not divide 128: forward and backward (with sinks) against the
    oracle -- padded heads and head groups must leave no trace."""
    import torch
    from mzoo_b200 import csa2_attn
    q, kv, _, main, idx, sk = _inputs(torch, cuda, 2, 160, H, 128, G=40, topk=32, seed=H, dup=True, holes=True,
                                      sinks=True)
    o, lse = csa2_attn.fwd(q, kv, main, idx, window=64, compress_ratio=4, sinks=sk)
    ref_o, ref_lse = A.attend(_np(q), _np(kv)[:, :, 0], window=64, main_kv=_np(main)[:, :, 0],
                              indices=idx.cpu().numpy(), sinks=_np(sk))
    _check(o, lse, ref_o, ref_lse, f"csa2 H{H}")
    do = _do(torch, cuda, q.shape, 3)
    dq, dkv, dmain, dsinks = csa2_attn.bwd(q, kv, main, idx, o, lse, do, window=64, compress_ratio=4, sinks=sk)
    ref = A.attend_bwd(_np(q), _np(kv)[:, :, 0], _np(do), window=64, main_kv=_np(main)[:, :, 0],
                       indices=idx.cpu().numpy(), sinks=_np(sk))
    _check_grad(dq, ref["dq"], f"csa2 dq H{H}")
    _check_grad(dkv[:, :, 0], ref["dkv"], f"csa2 dkv H{H}")
    _check_grad(dmain[:, :, 0], ref["dmain"], f"csa2 dmain H{H}")
    _check_grad(dsinks, ref["dsinks"], f"csa2 dsinks H{H}")
