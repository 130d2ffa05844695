"""Sliding-window shared-latent MQA with mzoo's ``swa_attn`` call signatures, on the
sm_100a kernel of ``csrc/attn_fwd.cu``.

Drop-in for ``src/mzoo/layers/attn/swa_attn``: ``fwd(q, kv, *, window, causal=True,
sinks=None) -> (o, lse)`` (``swa_attn/fwd.py:178``).  ``window`` counts the query itself
(``t - window + 1 <= k <= t``); ``window >= S`` is plain causal; ``causal=False`` is
rejected like the reference.  Additive keyword: ``v`` -- a distinct value tensor
[B,S,1,D] (the reference is K == V only; BASELINE config 5 quantises K and V
differently).
"""

import torch

from ._attn_common import check_mqa, run_bwd, run_fwd


def fwd(q: torch.Tensor, kv: torch.Tensor, *, window: int, causal: bool = True, sinks: torch.Tensor | None = None,
        v: torch.Tensor | None = None, softmax_scale: float | None = None):
    """q bf16 [B,S,H,D], kv bf16 [B,S,1,D] -> (o bf16 [B,S,H,D], lse fp32 [B,H,S])."""
    assert causal, "swa_attn is causal-only: a non-causal sliding window is not a model shape"
    assert isinstance(window, int) and window >= 1, f"window must be a positive int, got {window!r}"
    B, S, H, D = check_mqa(q, kv, "swa_attn")
    if sinks is not None:
        assert sinks.shape == (H,), f"sinks must be [H]={H}, got {tuple(sinks.shape)}"
        sinks = sinks.detach().float().contiguous()
    if v is not None:
        assert v.shape == kv.shape and v.dtype == torch.bfloat16, "v must match kv"
        v = v.contiguous()
    scale = softmax_scale if softmax_scale is not None else D**-0.5
    return run_fwd(q.contiguous(), kv.contiguous(), v, None, None, sinks, min(window, S), scale)


def bwd(q, kv, o, lse, do, *, window: int, causal: bool = True, sinks=None, cfg=None, splits=None, v=None,
        softmax_scale: float | None = None):
    """``swa_attn/bwd.py:79``: -> (dq bf16 [B,S,H,D], dkv bf16 [B,S,1,D], dsinks fp32 [H] or
    None).  With a distinct ``v`` the second output is dK and a fourth, dV, is appended.
    ``cfg`` / ``splits`` (the reference's tile and split-count knobs) are accepted and
    ignored: the kernel owns its tiling."""
    assert causal, "swa_attn is causal-only"
    assert q.shape == o.shape == do.shape, "shape mismatch"
    assert isinstance(window, int) and window >= 1, f"window must be a positive int, got {window!r}"
    B, S, H, D = check_mqa(q, kv, "swa_attn")
    assert D in (64, 96, 128, 256), f"swa_attn backward supports head dim 64 / 96 / 128 / 256, got {D}"
    assert v is None or D <= 128, "a separate v needs head dim <= 128 in backward"
    scale = softmax_scale if softmax_scale is not None else D**-0.5
    dq, dk, dv, _, dsinks = run_bwd(q.contiguous(), kv.contiguous(), None if v is None else v.contiguous(), None,
                                    None, o.contiguous(), lse.contiguous(), do.contiguous(), sinks, min(window, S),
                                    scale)
    return (dq, dk, dsinks) if v is None else (dq, dk, dsinks, dv)


class _Attn(torch.autograd.Function):
    """``swa_attn/attn.py:16``: saves q, kv (, v), o, lse (, sinks); recomputes in backward."""

    @staticmethod
    def forward(ctx, q, kv, window, causal, sinks, v, softmax_scale):
        o, lse = fwd(q, kv, window=window, causal=causal, sinks=sinks, v=v, softmax_scale=softmax_scale)
        ctx.save_for_backward(q, kv, o, lse, sinks if sinks is not None else q.new_empty(0),
                              v if v is not None else q.new_empty(0))
        ctx.window, ctx.causal, ctx.has_sinks, ctx.has_v, ctx.scale = window, causal, sinks is not None, \
            v is not None, softmax_scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, kv, o, lse, sinks, v = ctx.saved_tensors
        res = bwd(q, kv, o, lse, do, window=ctx.window, causal=ctx.causal,
                  sinks=sinks if ctx.has_sinks else None, v=v if ctx.has_v else None, softmax_scale=ctx.scale)
        dsinks = res[2] if ctx.has_sinks else None
        dv = res[3] if ctx.has_v else None
        return res[0], res[1], None, None, dsinks, dv, None


def attn(q: torch.Tensor, kv: torch.Tensor, *, window: int, causal: bool = True, sinks: torch.Tensor | None = None,
         v: torch.Tensor | None = None, softmax_scale: float | None = None) -> torch.Tensor:
    """``swa_attn/attn.py:33``: differentiable sliding-window attention -> o [B,S,H,D]."""
    return _Attn.apply(q, kv, window, causal, sinks, v, softmax_scale)
