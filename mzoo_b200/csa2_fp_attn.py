"""Window + top-k gathered shared-latent MQA over the quantised KV caches: the
``csa2_fp_attn`` of ``tickets/0010-csa2-fp-cache.md`` with ``csa2_attn``'s call shapes.

The window cache arrives as e4m3 codes + ue8m0 bytes per 32 channels, the main cache as
packed e2m1 + e4m3 bytes per 16 channels (``mzoo_b200.kvcache``).  Numerics do not move: the
attention sees exactly the bf16 values of the model's fake quantisers, through
``csa2_attn``'s kernels (same inputs, same numbers); the backward recomputes the same
dequantised tiles and passes the cache gradients straight through (STE, scales
stop-gradiented), the ticket's semantics.

Where the dequantisation happens: one fused unpack pass per cache per call
(``csrc/kvcache.cu``), not inside the attention kernels' tile loads.  At the training
shapes the unpacked caches are a few MB (S x D x 2 bytes for the window, G x D x 2 for the
main cache) and stay in L2 for the attention that follows, so the pass costs one read of
the packed bytes and one L2-resident write; the gathered reads of the main cache hit L2
either way.  ``tests/test_kvcache.py`` checks the outputs and gradients equal ``csa2_attn``
on the dequantised tensors bit for bit.
"""

import torch

from . import csa2_attn
from .kvcache import pack_main, pack_window, unpack_main, unpack_window


def _dequant(kv_codes, kv_scales, main_codes, main_scales):
    kv = unpack_window(kv_codes, kv_scales)      # [B,S,1,D]
    main = unpack_main(main_codes, main_scales)  # [B,G,1,D]
    return kv, main


def fwd(q: torch.Tensor, kv_codes: torch.Tensor, kv_scales: torch.Tensor, main_codes: torch.Tensor,
        main_scales: torch.Tensor, indices: torch.Tensor, *, window: int, compress_ratio: int, causal: bool = True,
        sinks: torch.Tensor | None = None, softmax_scale: float | None = None):
    """q bf16 [B,S,H,D]; window cache codes [B,S,1,D] + scales [B,S,1,D/32]; main cache
    codes [B,G,1,D/2] + scales [B,G,1,D/16]; indices [B,S,topk] -> (o bf16 [B,S,H,D],
    lse fp32 [B,H,S])."""
    kv, main = _dequant(kv_codes, kv_scales, main_codes, main_scales)
    return csa2_attn.fwd(q, kv, main, indices, window=window, compress_ratio=compress_ratio, causal=causal,
                         sinks=sinks, softmax_scale=softmax_scale)


def bwd(q, kv_codes, kv_scales, main_codes, main_scales, indices, o, lse, do, *, window: int, compress_ratio: int,
        causal: bool = True, sinks=None, softmax_scale: float | None = None):
    """-> (dq, dkv [B,S,1,D], dmain [B,G,1,D], dsinks): gradients w.r.t. the dequantised
    caches, i.e. the straight-through gradients of the latents the caches were packed from."""
    kv, main = _dequant(kv_codes, kv_scales, main_codes, main_scales)
    return csa2_attn.bwd(q, kv, main, indices, o, lse, do, window=window, compress_ratio=compress_ratio,
                         causal=causal, sinks=sinks, softmax_scale=softmax_scale)


class _Attn(torch.autograd.Function):
    """QAT form: bf16 latents in, packed into the cache formats, attention on the stored
    values, gradients straight through to the latents."""

    @staticmethod
    def forward(ctx, q, kv, main_kv, indices, window, compress_ratio, sinks, softmax_scale):
        kc, ks = pack_window(kv)
        mc, ms = pack_main(main_kv)
        o, lse = fwd(q, kc, ks, mc, ms, indices, window=window, compress_ratio=compress_ratio, sinks=sinks,
                     softmax_scale=softmax_scale)
        ctx.save_for_backward(q, kc, ks, mc, ms, indices, o, lse, *(() if sinks is None else (sinks,)))
        ctx.window, ctx.ratio, ctx.scale = window, compress_ratio, softmax_scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, kc, ks, mc, ms, indices, o, lse, *rest = ctx.saved_tensors
        dq, dkv, dmain, dsinks = bwd(q, kc, ks, mc, ms, indices, o, lse, do, window=ctx.window,
                                     compress_ratio=ctx.ratio, sinks=rest[0] if rest else None,
                                     softmax_scale=ctx.scale)
        return dq, dkv, dmain, None, None, None, dsinks, None


def attn(q: torch.Tensor, kv: torch.Tensor, main_kv: torch.Tensor, indices: torch.Tensor, *, window: int,
         compress_ratio: int, sinks: torch.Tensor | None = None, softmax_scale: float | None = None) -> torch.Tensor:
    """Differentiable attention over caches packed from the bf16 latents ``kv [B,S,1,D]``
    and ``main_kv [B,G,1,D]`` (the model's fake-quantised window and compressed caches)."""
    return _Attn.apply(q, kv, main_kv, indices, window, compress_ratio, sinks, softmax_scale)
