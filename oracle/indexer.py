"""Lightning-indexer oracle (numpy) -- test infrastructure, not the product.

Two restatements:

1. ``scores_ref`` / ``topk_ref`` -- ``golden_ref.indexer_scores`` (golden_ref.py:213-227)
   and ``golden_ref.topk_indices`` (golden_ref.py:230-243) in float32, pinned against the
   reference's own outputs in ``tests/golden/indexer.npz``.  ``topk_ref`` breaks ties by
   the lower index (the reference leaves tie order to ``torch.topk``).

2. ``canonical_scores`` / ``canonical_topk`` -- the exact definition the CUDA top-k
   selects against (``score = sum_h w_h relu(q_h . k) s_q s_k``):

       c_h   = w_h * sq_h                           (fp64, exact)
       dot_h = sum_i q_hi * k_i                     (fp64; exact for e4m3 codes in any
                                                     order, sequential for bf16)
       acc   = ((c_0 max(dot_0,0) + c_1 max(dot_1,0)) + ...)   (fp64, h ascending,
                                                     each product and sum rounded)
       score = (acc * sk) * scale                   (fp64)

   masked to -inf where ``t >= (q_offset + s + 1) // ratio`` (absolute positions,
   ``archs/dsv4/modeling_deepseek_v41.py:555-556``), top-k by (score desc, index asc),
   written ascending and -1 padded.
"""

import numpy as np


def visible(s: np.ndarray, ratio: int, q_offset: int, T: int) -> np.ndarray:
    v = (q_offset + s + 1) // ratio
    return np.clip(v, 0, T)


def scores_ref(q: np.ndarray, k: np.ndarray, w: np.ndarray, ratio: int, q_offset: int = 0) -> np.ndarray:
    """float32 ``indexer_scores``: q [B,S,Hi,Di], k [B,T,Di], w [B,S,Hi] -> [B,S,T]."""
    q, k, w = (np.asarray(x, np.float32) for x in (q, k, w))
    di = q.shape[-1]
    raw = np.maximum(np.einsum("bshd,btd->bsht", q, k), 0) * np.float32(di**-0.5)
    sc = (raw * w[..., None]).sum(axis=2, dtype=np.float32)
    S, T = q.shape[1], k.shape[1]
    vis = np.arange(T)[None, :] < visible(np.arange(S), ratio, q_offset, T)[:, None]
    return np.where(vis[None], sc, -np.inf).astype(np.float32)


def topk_ref(scores: np.ndarray, topk: int) -> np.ndarray:
    """``topk_indices``: per row the topk largest finite entries (ties -> lower index),
    -1 for -inf picks and for topk > T.  Returned sorted ascending for comparison."""
    B, S, T = scores.shape
    out = np.full((B, S, topk), -1, np.int64)
    kept = min(topk, T)
    for b in range(B):
        for s in range(S):
            row = scores[b, s]
            order = np.lexsort((np.arange(T), -row.astype(np.float64)))[:kept]
            picks = np.sort(order[np.isfinite(row[order])])
            out[b, s, :len(picks)] = picks
    return out


def _dots_fp64(qc: np.ndarray, kb: np.ndarray, exact_any_order: bool) -> np.ndarray:
    """[s,Hi,Di] x [T,Di] -> [s,Hi,T] in float64."""
    if exact_any_order:
        return np.einsum("shd,td->sht", qc, kb, optimize=True)
    acc = np.zeros((qc.shape[0], qc.shape[1], kb.shape[0]), np.float64)
    for i in range(qc.shape[-1]):
        acc = acc + qc[:, :, i, None] * kb[None, None, :, i]
    return acc


def canonical_scores(q: np.ndarray, k: np.ndarray, w: np.ndarray, sq, sk, ratio: int, q_offset: int = 0,
                     scale: float = 1.0, fp8: bool = True, chunk: int = 64) -> np.ndarray:
    """Exact-definition scores as float64 [B,S,T] (see module docstring).  ``q``/``k`` are
    the element values (e4m3 grid values or bf16 values) as float arrays; ``sq``/``sk``
    may be None (= 1)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    B, S, Hi, _ = q.shape
    T = k.shape[1]
    w64 = np.asarray(w, np.float32).astype(np.float64)
    c = w64 * (np.asarray(sq, np.float32).astype(np.float64) if sq is not None else 1.0)
    skd = np.asarray(sk, np.float32).astype(np.float64) if sk is not None else np.ones((B, T))
    scale64 = float(np.float32(scale))
    out = np.empty((B, S, T), np.float64)
    for b in range(B):
        for s0 in range(0, S, chunk):
            s1 = min(S, s0 + chunk)
            dots = _dots_fp64(q[b, s0:s1], k[b], fp8)
            acc = np.zeros((s1 - s0, T), np.float64)
            for h in range(Hi):
                acc = acc + c[b, s0:s1, h, None] * np.maximum(dots[:, h, :], 0.0)
            out[b, s0:s1] = (acc * skd[b][None, :]) * scale64
    vis = np.arange(T)[None, :] < visible(np.arange(S), ratio, q_offset, T)[:, None]
    return np.where(vis[None], out, -np.inf)


def canonical_topk(scores64: np.ndarray, topk: int, ratio: int, q_offset: int = 0) -> np.ndarray:
    """Top-k of canonical scores: ascending indices, -1 padded (int32 [B,S,topk])."""
    B, S, T = scores64.shape
    out = np.full((B, S, topk), -1, np.int32)
    vis = visible(np.arange(S), ratio, q_offset, T)
    for b in range(B):
        for s in range(S):
            v = int(vis[s])
            if v <= topk:
                out[b, s, :v] = np.arange(v)
                continue
            row = scores64[b, s, :v]
            order = np.lexsort((np.arange(v), -row))[:topk]
            out[b, s] = np.sort(order)
    return out


def bound_factors(q: np.ndarray, k: np.ndarray, w, sq, sk, scale: float = 1.0):
    """A_s = sum_h |w sq| ||q_h||_2 and B_t = |scale| sk_t ||k_t||_2 -- the factors of the
    fp32-score error bound the CUDA top-k uses (delta = eps * A_s * max_t B_t)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    c = np.abs(np.asarray(w, np.float64) * (np.asarray(sq, np.float64) if sq is not None else 1.0))
    A = (c * np.sqrt((q * q).sum(-1))).sum(-1)
    skd = np.asarray(sk, np.float64) if sk is not None else 1.0
    Bt = abs(scale) * np.abs(skd) * np.sqrt((k * k).sum(-1))
    return A, Bt


def scores_bwd_ref(q, k, w, dl, ratio: int, q_offset: int = 0, scale: float | None = None):
    """Gradients of ``indexer_scores`` (``indexer/bwd.py:4-22`` closed form) in float64:
    with r = q.k, d = dl * scale on visible keys (0 elsewhere, whatever dl holds there):
    dw = sum_t relu(r) d, dr = d w [r > 0], dq = sum_t dr k, dk = sum_{s,h} dr q."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    w = np.asarray(w, np.float64)
    dl = np.asarray(dl, np.float64)
    B, S, Hi, Di = q.shape
    T = k.shape[1]
    scale = Di**-0.5 if scale is None else scale
    vis = np.arange(T)[None, :] < visible(np.arange(S), ratio, q_offset, T)[:, None]
    d = np.where(vis[None], dl, 0.0) * scale
    r = np.einsum("bshd,btd->bsht", q, k)
    dw = (np.maximum(r, 0) * d[:, :, None, :]).sum(-1)
    dr = d[:, :, None, :] * w[..., None] * (r > 0)
    dq = np.einsum("bsht,btd->bshd", dr, k)
    dk = np.einsum("bsht,bshd->btd", dr, q)
    return dq, dk, dw
