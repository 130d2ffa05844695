"""Quantised KV-cache storage of the DeepSeek-V4.1 attention (the formats fixed in
``src/mzoo/layers/attn/csa_attn/README.md:215-235`` and ``tickets/0010-csa2-fp-cache.md``).

- window cache: e4m3 codes ``[..., D]`` + one ue8m0 byte per 32 channels ``[..., D/32]``
  (scale ``2**(byte - 127)``) -- the model's ``_fake_quant_fp8_block(x, 32)``;
- main (compressed) cache: e2m1 codes two per byte, low nibble first ``[..., D/2]`` + one
  e4m3 byte per 16 channels ``[..., D/16]`` -- ``_fake_quant_fp4_block(x, 16,
  e4m3_scales=True)`` (``archs/dsv4/modeling_deepseek_v41.py:359-402, :668-683``).

``unpack_*(pack_*(x))`` equals those fake quantisers bit for bit (``tests/test_kvcache.py``
against fixtures from the model's own functions).  One CUDA pass each way
(``csrc/kvcache.cu``); the attention on the packed caches is ``mzoo_b200.csa2_fp_attn``.
"""

import torch

from . import ops


def _rows(x: torch.Tensor, block: int) -> tuple:
    assert x.dtype == torch.bfloat16, f"the caches hold bf16 latents, got {x.dtype}"
    D = x.shape[-1]
    assert D % block == 0, f"D={D} must be a multiple of {block}"
    return x.reshape(-1, D).contiguous(), D


def pack_window(x: torch.Tensor) -> tuple:
    """bf16 ``[..., D]`` -> (e4m3 codes uint8 ``[..., D]``, ue8m0 scale bytes ``[..., D/32]``)."""
    flat, D = _rows(x, 32)
    codes, scales = ops.kv_pack(flat, 8)
    return codes.view(*x.shape[:-1], D), scales.view(*x.shape[:-1], D // 32)


def unpack_window(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """(codes ``[..., D]``, scales ``[..., D/32]``) -> bf16 ``[..., D]``."""
    D = codes.shape[-1]
    out = ops.kv_unpack(codes.reshape(-1, D).contiguous(), scales.reshape(-1, D // 32).contiguous(), D, 8)
    return out.view(*codes.shape[:-1], D)


def pack_main(x: torch.Tensor) -> tuple:
    """bf16 ``[..., D]`` -> (packed e2m1 uint8 ``[..., D/2]``, e4m3 scale bytes ``[..., D/16]``)."""
    flat, D = _rows(x, 16)
    codes, scales = ops.kv_pack(flat, 4)
    return codes.view(*x.shape[:-1], D // 2), scales.view(*x.shape[:-1], D // 16)


def unpack_main(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """(packed ``[..., D/2]``, scales ``[..., D/16]``) -> bf16 ``[..., D]``."""
    D = codes.shape[-1] * 2
    out = ops.kv_unpack(codes.reshape(-1, D // 2).contiguous(), scales.reshape(-1, D // 16).contiguous(), D, 4)
    return out.view(*codes.shape[:-1], D)
