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

from ._attn_common import check_mqa, run_fwd


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
