"""QK prologue oracle (numpy) -- test infrastructure, not the product.

Restates the model's RMSNorm followed by its interleaved-pair RoPE
(``archs/dsv4/modeling_deepseek_v41.py:49-63`` ``DeepseekV41RMSNorm.forward`` and
``:405-425`` ``apply_rotary_pos_emb``; composed as ``layers/attn/norm_rope.py:37-44``
``qk_norm_rope_eager``), in float32 with the same rounding points for bf16 inputs:

    h = x (fp32);  rstd = 1 / sqrt(mean(h^2) + eps);  xn = dtype(h * rstd)
    y = dtype(w * xn)                                   (product in fp32, one rounding)
    nope channels pass, each (even, odd) pair of the trailing rope_dim channels:
      y_e' = dtype(e*cos - o*sin), y_o' = dtype(e*sin + o*cos)   (fp32, each product rounded)

and the gradients of that composition in closed form (``norm_rope.py:121-128``): the rope
inverse-rotates dy to dxn, g = w * dxn, dx = rstd * (g - x * rstd^2 * mean(g * x)),
dw = sum over rows of dxn * x * rstd.  Pinned against the model's own modules in
``tests/golden/norm_rope.npz`` (``tests/test_norm_rope.py``).
"""

import numpy as np

from .quant import bf16_to_f32, f32_to_bf16


def _round(v: np.ndarray, dtype: str) -> np.ndarray:
    v = np.asarray(v, np.float32)
    return bf16_to_f32(f32_to_bf16(v)) if dtype == "bf16" else v


def norm_rope_fwd(x, w, cos, sin, eps: float = 1e-6, dtype: str = "f32"):
    """x [B,S,H,D] (values; bf16 values as float32 when dtype == "bf16"), w [D], cos / sin
    [B,S,rd/2] float32 -> (out [B,S,H,D] float32 values, rstd [B,S,H] float32)."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    D = x.shape[-1]
    rd = cos.shape[-1] * 2
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    rstd = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    xn = _round(x * rstd, dtype)
    y = _round(w * xn, dtype)
    out = y.copy()
    if rd:
        c = np.asarray(cos, np.float32)[:, :, None, :]
        s = np.asarray(sin, np.float32)[:, :, None, :]
        e, o = y[..., D - rd::2], y[..., D - rd + 1::2]
        out[..., D - rd::2] = _round((e * c).astype(np.float32) - (o * s).astype(np.float32), dtype)
        out[..., D - rd + 1::2] = _round((e * s).astype(np.float32) + (o * c).astype(np.float32), dtype)
    return out, rstd[..., 0]


def norm_rope_bwd(x, w, cos, sin, dy, eps: float = 1e-6):
    """Closed-form gradients (float64) of the fp32 composition: -> (dx [B,S,H,D], dw [D])."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    dy = np.asarray(dy, np.float64)
    D = x.shape[-1]
    rd = cos.shape[-1] * 2
    rstd = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    dxn = dy.copy()
    if rd:
        c = np.asarray(cos, np.float64)[:, :, None, :]
        s = np.asarray(sin, np.float64)[:, :, None, :]
        e, o = dy[..., D - rd::2], dy[..., D - rd + 1::2]
        dxn[..., D - rd::2] = e * c + o * s
        dxn[..., D - rd + 1::2] = o * c - e * s
    g = w * dxn
    dot = np.mean(g * x, axis=-1, keepdims=True)
    dx = rstd * (g - x * rstd * rstd * dot)
    dw = (dxn * x * rstd).reshape(-1, D).sum(0)
    return dx, dw
