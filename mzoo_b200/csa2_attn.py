"""Window + top-k gathered shared-latent MQA with mzoo's ``csa2_attn`` call signatures, on
the sm_100a kernel of ``csrc/attn_fwd.cu``.

Drop-in for ``src/mzoo/layers/attn/csa2_attn``: ``fwd(q, kv, main_kv, indices, *, window,
compress_ratio, causal=True, sinks=None) -> (o, lse)`` (``csa2_attn/fwd.py:238``).  As in
the reference, ``compress_ratio`` is documentation only (group-causality lives in
``indices``), an index outside ``[0, G)`` is an empty slot, duplicates count twice, and
``G == 0`` / ``topk == 0`` reduce to ``swa_attn``.
"""

import torch

from ._attn_common import check_mqa, run_bwd_groups, run_fwd_groups


def fwd(q: torch.Tensor, kv: torch.Tensor, main_kv: torch.Tensor, indices: torch.Tensor, *, window: int,
        compress_ratio: int, causal: bool = True, sinks: torch.Tensor | None = None,
        softmax_scale: float | None = None):
    """q bf16 [B,S,H,D], kv bf16 [B,S,1,D], main_kv bf16 [B,G,1,D], indices int32/int64
    [B,S,topk] -> (o bf16 [B,S,H,D], lse fp32 [B,H,S])."""
    assert causal, "csa2_attn is causal-only: a non-causal sliding window is not a model shape"
    assert isinstance(window, int) and window >= 1, f"window must be a positive int, got {window!r}"
    assert isinstance(compress_ratio, int) and compress_ratio >= 1, \
        f"compress_ratio must be a positive int, got {compress_ratio!r}"
    B, S, H, D = check_mqa(q, kv, "csa2_attn", any_heads=True)
    G = main_kv.shape[1]
    assert main_kv.shape == (B, G, 1, D), f"main_kv must be [B, G, 1, D], got {tuple(main_kv.shape)}"
    assert indices.dtype in (torch.int32, torch.int64), f"indices must be int32/int64, got {indices.dtype}"
    assert indices.dim() == 3 and indices.shape[:2] == (B, S), \
        f"indices must be [B, S, topk]=[{B}, {S}, *], got {tuple(indices.shape)}"
    if sinks is not None:
        assert sinks.shape == (H,), f"sinks must be [H]={H}, got {tuple(sinks.shape)}"
        sinks = sinks.detach().float().contiguous()
    scale = softmax_scale if softmax_scale is not None else D**-0.5
    main = main_kv.contiguous() if G else None
    idx = indices.to(torch.int32).contiguous() if (G and indices.shape[2]) else None
    return run_fwd_groups(q.contiguous(), kv.contiguous(), None, main, idx, sinks, min(window, S), scale)


def bwd(q, kv, main_kv, indices, o, lse, do, *, window: int, compress_ratio: int, causal: bool = True, sinks=None,
        cfg=None, splits=None, scatter: str = "atomic", softmax_scale: float | None = None):
    """``csa2_attn/bwd.py:67``: -> (dq [B,S,H,D], dkv [B,S,1,D], dmain_kv [B,G,1,D],
    dsinks [H] or None).  ``dmain_kv`` is accumulated with fp32 atomics (not bitwise
    reproducible run to run, like the reference).  ``cfg`` / ``splits`` are accepted and
    ignored; ``scatter`` must be "atomic" (the reference's other values are its bench
    ablations)."""
    assert causal, "csa2_attn is causal-only"
    assert scatter == "atomic", "only the atomic scatter is a real gradient"
    assert q.shape == o.shape == do.shape, "shape mismatch"
    assert isinstance(window, int) and window >= 1, f"window must be a positive int, got {window!r}"
    B, S, H, D = check_mqa(q, kv, "csa2_attn", any_heads=True)
    assert D in (64, 96, 128, 256), f"csa2_attn backward supports head dim 64 / 96 / 128 / 256, got {D}"
    G = main_kv.shape[1]
    scale = softmax_scale if softmax_scale is not None else D**-0.5
    main = main_kv.contiguous() if G else None
    idx = indices.to(torch.int32).contiguous() if (G and indices.shape[2]) else None
    dq, dkv, _, dmain, dsinks = run_bwd_groups(q.contiguous(), kv.contiguous(), None, main, idx, o.contiguous(),
                                        lse.contiguous(), do.contiguous(), sinks, min(window, S), scale)
    if dmain is None:
        dmain = torch.zeros_like(main_kv)
    return dq, dkv, dmain, dsinks


class _Attn(torch.autograd.Function):
    """``csa2_attn/attn.py:20``: saves (q, kv, main_kv, indices, o, lse[, sinks])."""

    @staticmethod
    def forward(ctx, q, kv, main_kv, indices, window, compress_ratio, causal, sinks, softmax_scale):
        o, lse = fwd(q, kv, main_kv, indices, window=window, compress_ratio=compress_ratio, causal=causal,
                     sinks=sinks, softmax_scale=softmax_scale)
        saved = (q, kv, main_kv, indices, o, lse)
        ctx.save_for_backward(*(saved if sinks is None else saved + (sinks,)))
        ctx.window, ctx.ratio, ctx.causal, ctx.scale = window, compress_ratio, causal, softmax_scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, kv, main_kv, indices, o, lse, *rest = ctx.saved_tensors
        dq, dkv, dmain, dsinks = bwd(q, kv, main_kv, indices, o, lse, do, window=ctx.window,
                                     compress_ratio=ctx.ratio, causal=ctx.causal, sinks=rest[0] if rest else None,
                                     softmax_scale=ctx.scale)
        return dq, dkv, dmain, None, None, None, None, dsinks, None


def attn(q: torch.Tensor, kv: torch.Tensor, main_kv: torch.Tensor, indices: torch.Tensor, *, window: int,
         compress_ratio: int, causal: bool = True, sinks: torch.Tensor | None = None,
         softmax_scale: float | None = None) -> torch.Tensor:
    """``csa2_attn/attn.py:40``: differentiable window + gathered attention -> o
    (``softmax_scale`` defaults to D**-0.5, as in ``fwd``)."""
    return _Attn.apply(q, kv, main_kv, indices, window, compress_ratio, causal, sinks, softmax_scale)
