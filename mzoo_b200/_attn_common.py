"""Host side shared by ``swa_attn`` and ``csa2_attn``: argument checks in the reference's
words and the call into ``mzb_attn_fwd`` (packed BSHD rows, K == V latent)."""

import torch

from . import ops
from ._lib import require_cuda

SUPPORTED_D = (64, 96, 128, 256)
# head dims the kernels tile directly; others are zero-padded to the next one on the host
# (zero channels add nothing to q.k, give zero output channels and zero gradients, so the
# padded run is the same attention; the softmax scale is passed from the original D)
KERNEL_D = {64: 64, 96: 128, 128: 128, 256: 256}


def _pad(x, D, Dk):
    if x is None or D == Dk:
        return x
    return torch.nn.functional.pad(x, (0, Dk - D)).contiguous()


def check_mqa(q: torch.Tensor, kv: torch.Tensor, what: str) -> tuple:
    """``swa_attn/fwd.py:167`` / ``csa2_attn/fwd.py:222``: q bf16 [B,S,H,D], kv [B,S,1,D]."""
    assert q.dtype == torch.bfloat16, f"expected bf16, got {q.dtype}"
    batch, seq_len, heads, dim = q.shape
    assert kv.shape == (batch, seq_len, 1, dim), \
        f"kv must be [B, S, 1, D]={(batch, seq_len, 1, dim)}, got {tuple(kv.shape)}"
    assert dim in SUPPORTED_D, f"unsupported head dim {dim}"
    assert 128 % heads == 0, f"{what} needs heads | 128 (packed 128-row query tiles), got H={heads}"
    return batch, seq_len, heads, dim


def run_fwd(q, kv, v, main_kv, idx, sinks, window, scale, check=False):
    require_cuda(q, kv, v, main_kv, idx, sinks)
    B, S, H, D = q.shape
    Dk = KERNEL_D[D]
    o, lse = ops.attn_fwd(_pad(q, D, Dk), _pad(kv, D, Dk), _pad(v, D, Dk), _pad(main_kv, D, Dk), idx, sinks, window,
                          float(scale), check)
    if Dk != D:
        o = o[..., :D].contiguous()
    return o, lse.view(B, S, H).permute(0, 2, 1).contiguous()


def run_bwd(q, kv, v, main_kv, idx, o, lse, do, sinks, window, scale, check=False):
    """-> (dq [B,S,H,D], dkv [B,S,1,D] (dK+dV when v is None, else dK), dv or None,
    dmain [B,G,1,D] or None, dsinks [H] or None)."""
    require_cuda(q, kv, v, main_kv, idx, o, lse, do)
    B, S, H, D = q.shape
    lse_packed = lse.permute(0, 2, 1).reshape(B, S * H).contiguous()  # [B,H,S] -> token-major rows
    G = main_kv.shape[1] if main_kv is not None else 0
    Dk = KERNEL_D[D]
    dq, dk, dv, dmain, delta = ops.attn_bwd(_pad(q, D, Dk), _pad(kv, D, Dk), _pad(v, D, Dk), _pad(main_kv, D, Dk), idx,
                                            _pad(o, D, Dk), lse_packed, _pad(do, D, Dk), window, float(scale), check)
    dv = dv if v is not None else None
    if Dk != D:
        dq, dk = dq[..., :D].contiguous(), dk[..., :D].contiguous()
        dv = dv[..., :D].contiguous() if dv is not None else None
        dmain = dmain[..., :D].contiguous() if G else dmain
    dsinks = None
    if sinks is not None:  # swa_attn/bwd.py, csa2_attn/bwd.py:123-127: a torch reduce over lse / delta
        d = delta[:, :S * H].view(B, S, H).permute(0, 2, 1)
        dsinks = -(torch.exp(sinks.detach().float().view(1, H, 1) - lse) * d).sum(dim=(0, 2))
    dmain_out = dmain.to(torch.bfloat16).view(B, G, 1, D) if G else None
    return dq, dk, dv, dmain_out, dsinks
