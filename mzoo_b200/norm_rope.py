"""Fused RMSNorm + RoPE prologue of q / kv with mzoo's call signature, on the sm_100a kernels
of ``csrc/norm_rope.cu``.

Drop-in for ``src/mzoo/layers/attn/norm_rope.py``: ``qk_norm_rope(x, weight, cos, sin, *,
eps=1e-6)`` (``norm_rope.py:227``) -- the model's ``DeepseekV41RMSNorm`` followed by
``apply_rotary_pos_emb`` (interleaved (even, odd) pairs of the trailing ``2 * cos.shape[-1]``
channels; leading channels pass through) in one pass over ``x``, differentiable: the
forward saves only x, weight, cos, sin and one fp32 rstd per row (``norm_rope.py:16-19``),
the backward recomputes the normed values.  x bf16 ``[B, S, H, D]`` (q) or ``[B, S, 1, D]``
(kv), weight bf16 ``[D]``, cos / sin fp32 ``[B, S, rope_dim / 2]``.
"""

import torch

from . import ops
from ._lib import require_cuda


def _prep(x, weight, cos, sin):
    require_cuda(x, weight, cos, sin)
    assert x.dim() == 4 and x.dtype == torch.bfloat16, f"x must be bf16 [B, S, H, D], got {x.dtype} {tuple(x.shape)}"
    B, S, H, D = x.shape
    assert weight.shape == (D,), f"weight must be [{D}], got {tuple(weight.shape)}"
    assert cos.shape == sin.shape and cos.shape[:2] == (B, S), \
        f"cos / sin must be [B, S, rope_dim / 2]=[{B}, {S}, *], got {tuple(cos.shape)}"
    rd = 2 * cos.shape[-1]
    assert rd <= D and (D - rd) % 2 == 0, f"rope_dim {rd} must fit the head dim {D}"
    x2 = x.contiguous().view(B * S * H, D)
    cs = cos.float().contiguous().view(B * S, -1) if rd else None
    sn = sin.float().contiguous().view(B * S, -1) if rd else None
    return x2, weight.to(torch.bfloat16).contiguous(), cs, sn, H


def fwd(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, eps: float = 1e-6):
    """-> (out bf16 like x, rstd fp32 [B*S*H])."""
    x2, w, cs, sn, H = _prep(x, weight, cos, sin)
    out, rstd = ops.norm_rope_fwd(x2, w, cs, sn, H, float(eps))
    return out.view(x.shape), rstd


def bwd(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rstd: torch.Tensor,
        dy: torch.Tensor):
    """-> (dx bf16 like x, dw fp32 [D]) for ``L(qk_norm_rope(x, weight, ...))`` given dL/dout."""
    x2, w, cs, sn, H = _prep(x, weight, cos, sin)
    assert dy.shape == x.shape, f"dy must be {tuple(x.shape)}, got {tuple(dy.shape)}"
    dx, dw = ops.norm_rope_bwd(x2, w, cs, sn, rstd.contiguous(), dy.to(torch.bfloat16).contiguous().view_as(x2), H)
    return dx.view(x.shape), dw


class _QKNormRoPE(torch.autograd.Function):
    """``norm_rope.py:199-224``: saves x, weight, cos, sin and rstd, no activation copy."""

    @staticmethod
    def forward(ctx, x, weight, cos, sin, eps):
        out, rstd = fwd(x, weight, cos, sin, eps=eps)
        ctx.save_for_backward(x, weight, cos, sin, rstd)
        return out

    @staticmethod
    def backward(ctx, dy):
        x, weight, cos, sin, rstd = ctx.saved_tensors
        dx, dw = bwd(x, weight, cos, sin, rstd, dy)
        return dx, dw.to(weight.dtype), None, None, None


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
                 eps: float = 1e-6) -> torch.Tensor:
    """Fused RMSNorm -> RoPE with backward (``norm_rope.py:227``)."""
    return _QKNormRoPE.apply(x, weight, cos, sin, eps)
