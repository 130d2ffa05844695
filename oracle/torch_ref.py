"""The reference's CPU arithmetic restated in torch float32 -- test infrastructure, not the
product.

pmonad/mzoo's CPU path for this hot path is plain PyTorch (``golden_ref.py``,
``archs/owlet1/quant.py``).  The reference itself cannot travel to the GPU host, so this
module restates the same float32 torch arithmetic, operation for operation, for two uses:
``bench.py``'s reference arm and CPU baseline time it on the host cores (all threads), and
``tests/`` pin it against the fixtures generated from the reference itself
(``tests/test_torch_ref.py``).

- ``attend``            ``golden_ref._attend`` (golden_ref.py:83-100), float32 path: one
                        matmul for the logits, an additive mask, logsumexp, softmax, matmul
- ``window_attention``  ``golden(level="window")`` (golden_ref.py:103-147, masks :67-82)
- ``gathered_attention`` ``_attend`` over each query token's gathered latent rows (the
                        576/512 FP8 latent of BASELINE configs 3 and 4), tokens batched with
                        a ``-inf`` bias on each token's unused key slots
- ``indexer_scores``    ``golden_ref.indexer_scores`` (golden_ref.py:213-227) with absolute
                        query positions and an explicit overall scale, chunked over queries
                        (as ``indexer/bench.py:31-43`` does)
- ``topk_indices``      ``golden_ref.topk_indices`` (golden_ref.py:230-243)
- ``pack_rows`` / ``unpack_rows``  576-channel latent <-> 672-byte FP8 rows (absmax/448
                        e4m3 per 64 channels, fp32 scales, bf16 rope)
- ``eager_sink_attention``  the DeepSeek-V4.1 layer's ``eager_attention_forward``
                        (modeling_deepseek_v41.py:581-611): shared K=V head, additive
                        mask, the per-head sink as one denominator-only logit
- ``qk_norm_rope``      the model's RMSNorm then interleaved-pair RoPE
                        (modeling_deepseek_v41.py:49-63, :405-425; ``norm_rope.py:37-44``)
- ``fake_quant_fp4_ocp`` / ``fake_quant_fp8_absmax``  the two rules BASELINE config 5
                        names, written like ``quant.py:49-86`` with the scale line swapped
"""

import torch

NEG_INF = float("-inf")


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None,
           scale: float | None = None) -> tuple:
    """q [B,H,S,D], k [B,Hk,T,D], v [B,Hk,T,Dv] (Hk broadcasts), mask an additive float32
    bias broadcastable to [B,H,S,T] or None -> (o [B,S,H,Dv], lse [B,H,S]) float32."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    logits = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if mask is not None:
        logits = logits + mask
    lse = torch.logsumexp(logits, dim=-1)
    probs = torch.softmax(logits, dim=-1)
    o = torch.matmul(probs, v.float())
    return o.transpose(1, 2), lse


def window_bias(S: int, window: int) -> torch.Tensor:
    """[S,S] additive bias: 0 where ``t - window < k <= t``, -inf elsewhere."""
    t = torch.arange(S).view(-1, 1)
    kk = torch.arange(S).view(1, -1)
    vis = (kk > t - window) & (kk <= t)
    return torch.zeros(S, S).masked_fill_(~vis, NEG_INF)


def window_attention(q: torch.Tensor, kv: torch.Tensor, window: int) -> tuple:
    """q [B,S,H,D], kv [B,S,1,D] (K == V) -> (o [B,S,H,D], lse [B,H,S]) float32."""
    S = q.shape[1]
    lat = kv.transpose(1, 2)
    return attend(q.transpose(1, 2), lat, lat, window_bias(S, window).view(1, 1, S, S))


def pack_rows(x: torch.Tensor) -> torch.Tensor:
    """[..., 576] float -> [..., 672] uint8 latent rows (torch's e4m3 and bf16 casts)."""
    lead = x.shape[:-1]
    xf = x.float()
    nope = xf[..., :512].reshape(*lead, 8, 64)
    amax = nope.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = (nope / scale.unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    rows = torch.empty(*lead, 672, dtype=torch.uint8)
    rows[..., :512] = codes.reshape(*lead, 512)
    rows[..., 512:544] = scale.contiguous().view(torch.uint8).reshape(*lead, 32)
    rows[..., 544:] = xf[..., 512:].to(torch.bfloat16).contiguous().view(torch.uint8).reshape(*lead, 128)
    return rows


def unpack_rows(rows: torch.Tensor) -> torch.Tensor:
    """[..., 672] uint8 latent rows -> [..., 576] float32: 512 e4m3 codes times their
    64-channel fp32 scale, then 64 bf16 rope channels."""
    lead = rows.shape[:-1]
    rows = rows.contiguous()
    scale = rows[..., 512:544].contiguous().view(torch.float32).reshape(*lead, 8, 1)
    nope = rows[..., :512].contiguous().view(torch.float8_e4m3fn).float().reshape(*lead, 8, 64) * scale
    rope = rows[..., 544:].contiguous().view(torch.bfloat16).float().reshape(*lead, 64)
    return torch.cat([nope.reshape(*lead, 512), rope], -1)


def gathered_attention(q: torch.Tensor, keys: torch.Tensor, counts: torch.Tensor, scale: float,
                       dv: int = 512) -> tuple:
    """q [n,H,D] (one query token each), keys [n,T,D] float32 (token i uses its first
    counts[i] rows; K = the rows, V = their first ``dv`` channels) -> (o [n,H,dv],
    lse [n,H])."""
    n, T = keys.shape[:2]
    bias = torch.zeros(n, T).masked_fill_(torch.arange(T).view(1, -1) >= counts.view(-1, 1), NEG_INF)
    # one shared key head: the H query heads are the rows of one [H, D] x [D, T] product per
    # token (``_attend`` with the heads on its query axis), so K is never copied per head
    o, lse = attend(q.unsqueeze(1), keys.unsqueeze(1), keys[..., :dv].unsqueeze(1), bias.view(n, 1, 1, T), scale)
    return o[:, :, 0], lse[:, 0]


def indexer_scores(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, ratio: int, q_offset: int = 0,
                   scale: float | None = None, chunk: int = 256) -> torch.Tensor:
    """q [B,S,Hi,Di], k [B,T,Di], w [B,S,Hi] -> float32 [B,S,T]:
    ``sum_h w relu(q_h . k) * scale``, -inf where ``t >= (q_offset + s + 1) // ratio``."""
    B, S, Hi, Di = q.shape
    T = k.shape[1]
    scale = Di ** -0.5 if scale is None else scale
    out = torch.empty(B, S, T)
    kf = k.float()
    for s0 in range(0, S, chunk):
        s1 = min(S, s0 + chunk)
        raw = torch.einsum("bshd,btd->bsht", q[:, s0:s1].float(), kf).relu_() * scale
        out[:, s0:s1] = (raw * w[:, s0:s1].float().unsqueeze(-1)).sum(dim=2)
    vis = torch.arange(T).view(1, -1) < ((torch.arange(S) + q_offset + 1) // ratio).view(-1, 1)
    return out.masked_fill_(~vis.unsqueeze(0), NEG_INF)


def topk_indices(scores: torch.Tensor, topk: int) -> torch.Tensor:
    """[..., T] float32 -> int64 [..., topk]: ``torch.topk(sorted=False)`` of the row, -1 for
    -inf picks and for topk > T."""
    T = scores.shape[-1]
    kk = min(topk, T)
    top = scores.topk(kk, dim=-1, sorted=False)
    idx = torch.where(top.values > NEG_INF, top.indices, torch.full_like(top.indices, -1))
    if kk < topk:
        idx = torch.cat([idx, idx.new_full((*idx.shape[:-1], topk - kk), -1)], -1)
    return idx


_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
# e2m1 rounding thresholds (quant.py:34-46): ties at 0.25 / 1.25 / 2.5 / 5.0 round down
# (strictly above), at 0.75 / 1.75 / 3.5 round up (at or above)
_THR = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
_TIES_UP = torch.tensor([False, True, False, True, False, True, False])


def fake_quant_fp4_ocp(x: torch.Tensor, block: int = 32) -> torch.Tensor:
    """OCP MXFP4 quant-dequant along the last axis: e8m0 scale 2^(floor(log2 amax) - 2)
    (1 for an all-zero block), elements saturated at +-6 and rounded onto e2m1."""
    n = x.shape[-1]
    xf = x.float().reshape(*x.shape[:-1], n // block, block)
    amax = xf.abs().amax(-1, keepdim=True)
    _, ex = torch.frexp(amax)                    # amax = m * 2^ex, m in [0.5, 1): floor(log2) = ex - 1
    e = (ex - 3).clamp(-127, 127).float()
    scale = torch.where(amax > 0, torch.exp2(e), torch.ones_like(amax))
    qv = (xf / scale).clamp(-6.0, 6.0)
    mag = qv.abs().unsqueeze(-1)
    code = torch.where(_TIES_UP, mag >= _THR, mag > _THR).sum(-1)
    y = torch.where(qv < 0, -_E2M1[code], _E2M1[code]) * scale
    return y.reshape(x.shape).to(x.dtype)


def fake_quant_fp8_absmax(x: torch.Tensor, block: int = 128) -> torch.Tensor:
    """FP8 e4m3 quant-dequant with a per-tile absmax scale (amax / 448, 1 when 0)."""
    n = x.shape[-1]
    xf = x.float().reshape(*x.shape[:-1], n // block, block)
    scale = xf.abs().amax(-1, keepdim=True) / 448.0
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    y = (xf / scale).clamp(-448, 448).to(torch.float8_e4m3fn).float() * scale
    return y.reshape(x.shape).to(x.dtype)


def qk_norm_rope(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 eps: float = 1e-6) -> torch.Tensor:
    """x [B,S,H,D], w [D], cos / sin [B,S,rd/2] -> RMSNorm (fp32 statistics, ``w * x.to(dtype)``)
    then RoPE on the trailing rd channels' (even, odd) pairs, in x's dtype."""
    dtype = x.dtype
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    y = w * h.to(dtype)
    rd = cos.shape[-1] * 2
    nope, rope = y[..., :-rd], y[..., -rd:]
    c, s = cos.unsqueeze(2), sin.unsqueeze(2)
    even, odd = rope[..., 0::2].float(), rope[..., 1::2].float()
    rot = torch.stack([even * c - odd * s, even * s + odd * c], dim=-1).flatten(-2)
    return torch.cat([nope, rot.to(dtype)], dim=-1)


def eager_sink_attention(q: torch.Tensor, kv: torch.Tensor, mask: torch.Tensor | None, sinks: torch.Tensor,
                         scaling: float) -> torch.Tensor:
    """q [B,H,S,D], kv [B,1,T,D] (K == V), additive mask [B,1,S,T] or None, sinks [H] ->
    o [B,S,H,D] float32: logits + mask, the sink column joined to the softmax and dropped
    (it only grows the denominator), probabilities times the shared V."""
    B, H, S, _ = q.shape
    logits = torch.matmul(q.float(), kv.float().transpose(2, 3)) * scaling
    if mask is not None:
        logits = logits + mask.float()
    sk = sinks.float().reshape(1, -1, 1, 1).expand(B, H, S, 1)
    combined = torch.cat([logits, sk], dim=-1)
    combined = combined - combined.max(dim=-1, keepdim=True).values
    probs = torch.softmax(combined, dim=-1)[..., :-1]
    return torch.matmul(probs, kv.float()).transpose(1, 2)
