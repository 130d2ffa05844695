"""Compressor producer-step oracle (numpy) -- test infrastructure, not the product.

Restates, after the two fp32 projections (``wkv``, ``wgate``), what
``DeepseekV41Compressor.forward`` (``src/mzoo/archs/dsv4/modeling_deepseek_v41.py:310-340``)
and its consumer (``:745-753``) do to one group of ``ratio`` consecutive tokens:

- pool (fp32): ``latent = sum_r kv_r * softmax_r(gate_r)`` per channel (``:338``), cast to
  bf16 (``:339``);
- ``DeepseekV41RMSNorm`` (``:58-63``): x fp32, ``x * rsqrt(mean(x^2) + eps)`` -> bf16, times
  the bf16 weight -> bf16.  This is the pre-RoPE latent the indexer consumes;
- ``apply_rotary_pos_emb`` (``:405-425``): adjacent (even, odd) pairs of the trailing
  ``rope_dim`` channels rotated in fp32 (``e*cos - o*sin``, ``e*sin + o*cos``, each product
  and sum rounded), cast to bf16;
- ``_fake_quant_fp4_block(rotated, 16, e4m3_scales=True)`` (``:753``): the compressed-cache
  entry.

At ``ratio == 1`` there is no gate: the latent is the projection cast to bf16, then normed.
Pinned against the reference's own module and functions in ``tests/golden/compressor.npz``.
Pool and variance are computed here in float64 and rounded once, so the bf16 latent can
differ from torch's fp32 evaluation by one bf16 unit where a value sits on a rounding
boundary; rope and fake quant are bit-exact given the same bf16 latent.
"""

import numpy as np

from . import quant as Q


def pool_ref(kv: np.ndarray, gate: np.ndarray | None, ratio: int) -> np.ndarray:
    """kv, gate fp32 [B, G*ratio, D] -> pooled fp32 [B, G, D] (gate None: the first G rows)."""
    B, N, D = kv.shape
    G = N // ratio
    if gate is None:
        return kv[:, :G].astype(np.float32)
    k = kv[:, :G * ratio].reshape(B, G, ratio, D).astype(np.float64)
    g = gate[:, :G * ratio].reshape(B, G, ratio, D).astype(np.float64)
    e = np.exp(g - g.max(axis=2, keepdims=True))
    w = e / e.sum(axis=2, keepdims=True)
    return (k * w).sum(axis=2).astype(np.float32)


def latent_ref(kv, gate, norm_w_bits: np.ndarray, eps: float, ratio: int) -> np.ndarray:
    """bf16 bits [B, G, D]: pooled, cast to bf16, RMS-normed, times the bf16 weight."""
    x = Q.bf16_to_f32(Q.f32_to_bf16(pool_ref(kv, gate, ratio))).astype(np.float64)
    var = (x * x).mean(axis=-1, keepdims=True)
    y = Q.f32_to_bf16((x / np.sqrt(var + eps)).astype(np.float32))
    w = Q.bf16_to_f32(norm_w_bits).astype(np.float32)
    return Q.f32_to_bf16((w * Q.bf16_to_f32(y)).astype(np.float32))


def rope_ref(latent_bits: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """bf16 bits [B, G, D] with the trailing 2*cos.shape[-1] channels rotated pairwise."""
    rd = 2 * cos.shape[-1]
    x = Q.bf16_to_f32(latent_bits)
    out = latent_bits.copy()
    e, o = x[..., -rd::2], x[..., -rd + 1::2]
    c, s = cos.astype(np.float32), sin.astype(np.float32)
    re = (e * c).astype(np.float32) - (o * s).astype(np.float32)
    ro = (e * s).astype(np.float32) + (o * c).astype(np.float32)
    rot = np.stack([re.astype(np.float32), ro.astype(np.float32)], axis=-1).reshape(*x.shape[:-1], rd)
    out[..., -rd:] = Q.f32_to_bf16(rot)
    return out


def cache_ref(latent_bits: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """bf16 bits: the compressed-cache entry (rotated, MXFP4 block 16 with e4m3 scales)."""
    return Q.fake_quant_fp4(rope_ref(latent_bits, cos, sin), 16, rule="e4m3", dtype="bf16")
