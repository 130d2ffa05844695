"""Shared-latent attention oracle (numpy) -- test infrastructure, not the product.

Restates ``golden_ref.golden`` (``src/mzoo/layers/attn/golden_ref.py:67-168``) for the
levels the hot path uses -- ``window`` and ``sparse`` -- plus its autograd gradients in
closed form, in float64.  Pinned against ``tests/golden/attention.npz`` (produced by the
reference itself).

Conventions (golden_ref.py:12-24): BSHD in/out; K == V latent [B,S,1,D] unless ``v`` is
given; window keeps keys ``t - W < k <= t``; sparse entries are exactly the listed
``indices`` (-1 = empty; duplicates kept, i.e. counted twice, like the kernels -- the
golden oracle itself deduplicates through a scatter mask, so tests of duplicates compare
against this form); sinks add one denominator-only logit per head; lse is natural-log
[B,H,S]; scale D**-0.5 unless given.
"""

import numpy as np


def _logits_keys(q, kv, main, idx, b, t, window):
    """Key rows (value rows) of query token t of batch b: window then gathered."""
    lo = max(0, t - window + 1)
    keys = [kv[b, lo:t + 1]]
    if main is not None and idx is not None:
        g = main.shape[1]
        sel = [int(i) for i in idx[b, t] if 0 <= i < g]
        if sel:
            keys.append(main[b, sel])
    return np.concatenate(keys, 0)


def attend(q, kv, *, window, v=None, main_kv=None, indices=None, sinks=None, scale=None):
    """q [B,S,H,D], kv [B,S,D] (or [B,S,1,D]), v like kv or None (= kv), main_kv [B,G,D]
    or None, indices [B,S,topk] or None, sinks [H] or None -> (o [B,S,H,D], lse [B,H,S])
    float64."""
    q = np.asarray(q, np.float64)
    kv = np.asarray(kv, np.float64).reshape(q.shape[0], q.shape[1], -1)
    vv = kv if v is None else np.asarray(v, np.float64).reshape(kv.shape)
    main = None if main_kv is None else np.asarray(main_kv, np.float64).reshape(q.shape[0], -1, q.shape[-1])
    B, S, H, D = q.shape
    scale = D**-0.5 if scale is None else scale
    o = np.zeros((B, S, H, D))
    lse = np.zeros((B, H, S))
    for b in range(B):
        for t in range(S):
            k = _logits_keys(q, kv, main, indices, b, t, window)
            vals = _logits_keys(q, vv, main, indices, b, t, window)
            z = q[b, t] @ k.T * scale  # [H, n]
            cols = [z]
            if sinks is not None:
                cols.append(np.asarray(sinks, np.float64)[:, None])
            zz = np.concatenate(cols, 1)
            m = zz.max(1, keepdims=True)
            e = np.exp(zz - m)
            l = e.sum(1, keepdims=True)
            p = e[:, :z.shape[1]] / l
            o[b, t] = p @ vals
            lse[b, :, t] = (m + np.log(l))[:, 0]
    return o, lse


def attend_bwd(q, kv, do, *, window, v=None, main_kv=None, indices=None, sinks=None, scale=None):
    """Gradients of ``attend`` (sum(o * do)) -> dict(dq, dk, dv, dmain, dsinks) float64.
    With K == V (v None) the kv gradient is dk + dv (returned as ``dkv``)."""
    q = np.asarray(q, np.float64)
    B, S, H, D = q.shape
    kv = np.asarray(kv, np.float64).reshape(B, S, D)
    vv = kv if v is None else np.asarray(v, np.float64).reshape(B, S, D)
    main = None if main_kv is None else np.asarray(main_kv, np.float64).reshape(B, -1, D)
    do = np.asarray(do, np.float64)
    scale = D**-0.5 if scale is None else scale
    dq = np.zeros_like(q)
    dk = np.zeros((B, S, D))
    dv = np.zeros((B, S, D))
    dmain = None if main is None else np.zeros_like(main)
    dsinks = None if sinks is None else np.zeros(H)
    for b in range(B):
        for t in range(S):
            lo = max(0, t - window + 1)
            nw = t + 1 - lo
            sel = []
            if main is not None and indices is not None:
                sel = [int(i) for i in indices[b, t] if 0 <= i < main.shape[1]]
            k = np.concatenate([kv[b, lo:t + 1]] + ([main[b, sel]] if sel else []), 0)
            vals = np.concatenate([vv[b, lo:t + 1]] + ([main[b, sel]] if sel else []), 0)
            z = q[b, t] @ k.T * scale
            zz = z if sinks is None else np.concatenate([z, np.asarray(sinks, np.float64)[:, None]], 1)
            m = zz.max(1, keepdims=True)
            e = np.exp(zz - m)
            pfull = e / e.sum(1, keepdims=True)
            p = pfull[:, :z.shape[1]]
            o = p @ vals
            g = do[b, t]  # [H, D]
            dp = g @ vals.T  # [H, n]
            delta = (g * o).sum(1, keepdims=True)
            ds = p * (dp - delta)  # [H, n]
            dq[b, t] = ds @ k * scale
            dkeys = ds.T @ q[b, t] * scale  # [n, D]
            dvals = p.T @ g
            dk[b, lo:t + 1] += dkeys[:nw]
            dv[b, lo:t + 1] += dvals[:nw]
            for i, gi in enumerate(sel):
                dmain[b, gi] += dkeys[nw + i] + dvals[nw + i]
            if sinks is not None:
                dsinks -= pfull[:, -1] * delta[:, 0]
    out = dict(dq=dq, dk=dk, dv=dv, dmain=dmain, dsinks=dsinks)
    if v is None:
        out["dkv"] = dk + dv
    return out
