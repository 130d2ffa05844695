"""Compressor producer step (DeepSeek-V4.1 CSA) on sm_100a kernels.

Replaces ``DeepseekV41Compressor.forward`` (``src/mzoo/archs/dsv4/modeling_deepseek_v41.py:318-340``)
and the compressed-cache write that follows it (``:745-753``):

- ``compressor_forward(hidden_states, wkv, wgate, norm_weight, compress_ratio, eps)`` ->
  the pre-RoPE latent ``[B, G, D]`` (the module's return value, without a cache layer:
  tokens past the last full group are dropped, ``first_group_position`` is 0);
- ``compress(kv, gate, norm_weight, compress_ratio, eps, cos=None, sin=None)`` -> ``(latent,
  cache)`` from the two fp32 projections, where ``cache`` (when ``cos`` / ``sin`` are
  given) is ``_fake_quant_fp4_block(apply_rotary_pos_emb(latent, cos, sin), 16,
  e4m3_scales=True)``, the entry the model stores in its compressed KV cache.

The projections are plain fp32 GEMMs (``torch.nn.functional.linear``, as the reference);
everything after them is one fused kernel (``csrc/compressor.cu``).  The model dtype is
bf16: the latent, the norm weight and the cache entry are bf16.
"""

import torch

from . import ops
from ._lib import require_cuda


def _aligned(t: torch.Tensor | None, n: int) -> torch.Tensor | None:
    if t is None:
        return None
    t = t.contiguous()
    return t if t.data_ptr() % n == 0 else t.clone()


def compress(kv: torch.Tensor, gate: torch.Tensor | None, norm_weight: torch.Tensor, compress_ratio: int,
             eps: float = 1e-6, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None) -> tuple:
    """kv, gate fp32 ``[B, G*ratio, D]`` (gate ``None`` at ratio 1); ``cos`` / ``sin``
    ``[B, G, rope_dim/2]``.  Returns ``(latent bf16 [B, G, D], cache bf16 [B, G, D] or None)``."""
    require_cuda(kv, gate, norm_weight, cos, sin)
    B, N, D = kv.shape
    ratio = int(compress_ratio)
    G = N // ratio
    kv = _aligned(kv[:, :G * ratio].float(), 16)
    if gate is not None:
        gate = _aligned(gate[:, :G * ratio].float(), 16)
    w = _aligned(norm_weight.to(torch.bfloat16), 8)
    rope = 0
    if cos is not None:
        assert sin is not None and cos.shape == sin.shape == (B, G, cos.shape[-1]), \
            f"cos / sin must be [B, G, rope_dim/2] = [{B}, {G}, r], got {tuple(cos.shape)}"
        rope = 2 * cos.shape[-1]
        cos, sin = cos.float().contiguous(), sin.float().contiguous()
    latent, cache = ops.compress(kv, gate, w, cos, sin, ratio, rope, float(eps))
    return latent, (cache if cos is not None else None)


def compressor_forward(hidden_states: torch.Tensor, wkv: torch.Tensor, wgate: torch.Tensor | None,
                       norm_weight: torch.Tensor, compress_ratio: int, eps: float = 1e-6) -> torch.Tensor:
    """The module's forward without a cache layer: ``[B, G, D]`` pre-RoPE latent (bf16)."""
    ratio = int(compress_ratio)
    usable = (hidden_states.shape[1] // ratio) * ratio
    h = hidden_states[:, :usable]
    if ratio == 1:  # no pooling: the projection in the model dtype
        kv = torch.nn.functional.linear(h, wkv.to(h.dtype)).float()
        return compress(kv, None, norm_weight, 1, eps)[0]
    hf = h.float()
    kv = torch.nn.functional.linear(hf, wkv.float())
    gate = torch.nn.functional.linear(hf, wgate.float())
    return compress(kv, gate, norm_weight, ratio, eps)[0]
