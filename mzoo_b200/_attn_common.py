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


def check_mqa(q: torch.Tensor, kv: torch.Tensor, what: str, any_heads: bool = False) -> tuple:
    """``swa_attn/fwd.py:167`` / ``csa2_attn/fwd.py:222``: q bf16 [B,S,H,D], kv [B,S,1,D].
    ``swa_attn`` needs H | 128 like the reference (``swa_attn/fwd.py:172``); ``csa2_attn``
    takes any H, as the reference does (``csa2_attn/fwd.py:65-67``), through head groups
    (``head_groups``)."""
    assert q.dtype == torch.bfloat16, f"expected bf16, got {q.dtype}"
    batch, seq_len, heads, dim = q.shape
    assert kv.shape == (batch, seq_len, 1, dim), \
        f"kv must be [B, S, 1, D]={(batch, seq_len, 1, dim)}, got {tuple(kv.shape)}"
    assert dim in SUPPORTED_D, f"unsupported head dim {dim}"
    assert heads >= 1, f"{what} needs at least one head"
    assert any_heads or 128 % heads == 0, f"{what} needs heads | 128 (packed 128-row query tiles), got H={heads}"
    return batch, seq_len, heads, dim


def head_groups(H: int) -> tuple:
    """The kernels pack (token, head) rows into 128-row query tiles, so a launch needs
    H | 128.  Other head counts run as launches of Hc heads each (Hc = the next power of two
    >= H up to 128, else 128), the last group zero-padded: a padded head has q = 0, o = 0,
    lse = 0 and dO = 0, so it adds nothing to any output or gradient.  -> (Hc, groups)."""
    if 128 % H == 0:
        return H, 1
    if H < 128:
        return 1 << (H - 1).bit_length(), 1
    return 128, -(-H // 128)


def _heads(x, h0, h1, H):
    """Heads [h0, h1) of x [..., H, D] (dim -2), zero-padded when h1 > H."""
    if x is None:
        return None
    part = x[..., h0:min(h1, H), :]
    if h1 > H:
        part = torch.nn.functional.pad(part, (0, 0, 0, h1 - H))
    return part.contiguous()


def run_fwd_groups(q, kv, v, main_kv, idx, sinks, window, scale, check=False):
    """``run_fwd`` for any head count (``head_groups``)."""
    B, S, H, D = q.shape
    Hc, ng = head_groups(H)
    if ng == 1 and Hc == H:
        return run_fwd(q, kv, v, main_kv, idx, sinks, window, scale, check)
    os_, ls_ = [], []
    for gi in range(ng):
        h0, h1 = gi * Hc, gi * Hc + Hc
        sk = None
        if sinks is not None:
            sk = torch.nn.functional.pad(sinks[h0:min(h1, H)], (0, max(0, h1 - H))).contiguous()
        o, lse = run_fwd(_heads(q, h0, h1, H), kv, v, main_kv, idx, sk, window, scale, check)
        os_.append(o)
        ls_.append(lse)
    return torch.cat(os_, 2)[:, :, :H].contiguous(), torch.cat(ls_, 1)[:, :H].contiguous()


def run_bwd_groups(q, kv, v, main_kv, idx, o, lse, do, sinks, window, scale, check=False):
    """``run_bwd`` for any head count: per-group dq / dsinks concatenated, the shared
    dkv / dv / dmain summed over the groups."""
    B, S, H, D = q.shape
    Hc, ng = head_groups(H)
    if ng == 1 and Hc == H:
        return run_bwd(q, kv, v, main_kv, idx, o, lse, do, sinks, window, scale, check)
    dqs, dss = [], []
    dk = dv = dmain = None
    for gi in range(ng):
        h0, h1 = gi * Hc, gi * Hc + Hc
        sk = None
        if sinks is not None:
            sk = torch.nn.functional.pad(sinks[h0:min(h1, H)], (0, max(0, h1 - H))).contiguous()
        lse_g = lse[:, h0:min(h1, H)]
        if h1 > H:
            lse_g = torch.nn.functional.pad(lse_g, (0, 0, 0, h1 - H))
        r = run_bwd(_heads(q, h0, h1, H), kv, v, main_kv, idx, _heads(o, h0, h1, H), lse_g.contiguous(),
                    _heads(do, h0, h1, H), sk, window, scale, check)
        dqs.append(r[0])
        dk = r[1].float() if dk is None else dk + r[1].float()
        if r[2] is not None:
            dv = r[2].float() if dv is None else dv + r[2].float()
        if r[3] is not None:
            dmain = r[3].float() if dmain is None else dmain + r[3].float()
        if r[4] is not None:
            dss.append(r[4])
    dq = torch.cat(dqs, 2)[:, :, :H].contiguous()
    ds = torch.cat(dss)[:H] if dss else None
    bf = lambda t: None if t is None else t.to(torch.bfloat16)
    return dq, bf(dk), bf(dv), bf(dmain), ds


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
