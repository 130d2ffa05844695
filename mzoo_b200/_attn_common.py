"""Host side shared by ``swa_attn`` and ``csa2_attn``: argument checks in the reference's
words and the call into ``mzb_attn_fwd`` (packed BSHD rows, K == V latent)."""

import torch

from . import _lib
from ._lib import call, ptr, require_cuda, stream_ptr

SUPPORTED_D = (64, 128, 256)


def check_mqa(q: torch.Tensor, kv: torch.Tensor, what: str) -> tuple:
    """``swa_attn/fwd.py:167`` / ``csa2_attn/fwd.py:222``: q bf16 [B,S,H,D], kv [B,S,1,D]."""
    assert q.dtype == torch.bfloat16, f"expected bf16, got {q.dtype}"
    batch, seq_len, heads, dim = q.shape
    assert kv.shape == (batch, seq_len, 1, dim), \
        f"kv must be [B, S, 1, D]={(batch, seq_len, 1, dim)}, got {tuple(kv.shape)}"
    assert dim in SUPPORTED_D, f"unsupported head dim {dim}"
    assert 128 % heads == 0, f"{what} needs heads | 128 (packed 128-row query tiles), got H={heads}"
    return batch, seq_len, heads, dim


def run_fwd(q, kv, v, main_kv, idx, sinks, window, scale, check=True):
    require_cuda(q, kv, v, main_kv, idx, sinks)
    B, S, H, D = q.shape
    dev = q.device
    o = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, S * H, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    G = main_kv.shape[1] if main_kv is not None else 0
    topk = idx.shape[2] if idx is not None else 0
    call("mzb_attn_fwd", ptr(q), ptr(kv), ptr(v), ptr(main_kv), ptr(idx), ptr(sinks), ptr(o), ptr(lse), B, S, H, D,
         window, G, topk, float(scale), ptr(err), stream_ptr(dev))
    if check and int(err.item()):
        raise _lib.MzbError(f"attn_fwd: device error code {int(err.item())}")
    return o, lse.view(B, S, H).permute(0, 2, 1).contiguous()
