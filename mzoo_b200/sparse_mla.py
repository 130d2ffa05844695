"""Sparse latent-MQA attention over FP8 KV rows (DeepSeek-V4.1 576/512 latent): prefill
forward and paged decode, on the sm_100a kernel of ``csrc/sparse_mla.cu``.

The reference (``src/mzoo/layers/attn/csa2_attn``) implements the same window + gathered
top-k attention for K == V latents with D <= 256 in bf16 (``csa2_attn/fwd.py:56-61``);
this module is its 576/512 FP8-cache form (BASELINE configs 3 and 4): K is the 576-dim
latent (512 no-rope channels stored e4m3 with one fp32 scale per 64 channels, 64 rope
channels bf16), V is its first 512 channels, scale ``576**-0.5`` by default.

KV rows are 672 bytes (``pack_kv``).  Semantics follow ``csa2_attn.fwd``: a causal window
of ``window`` raw tokens ending at the query (itself included), then the listed
compressed entries (``-1`` / out-of-range = empty, duplicates count twice), one softmax,
lse in natural log.
"""

import torch

from . import ops
from ._lib import require_cuda

H, DQK, DV, ROW_BYTES = 128, 576, 512, 672


def pack_kv(kv: torch.Tensor) -> torch.Tensor:
    """[..., 576] float -> [..., 672] uint8 rows: e4m3 no-rope codes with an absmax/448
    fp32 scale per 64 channels, then the scales, then the bf16 rope channels."""
    require_cuda(kv)
    assert kv.shape[-1] == DQK, f"latent must be {DQK}-dim, got {kv.shape[-1]}"
    lead = kv.shape[:-1]
    x = kv.float()
    nope = x[..., :512].reshape(*lead, 8, 64)
    amax = nope.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = (nope / scale.unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    rows = torch.empty(*lead, ROW_BYTES, dtype=torch.uint8, device=kv.device)
    rows[..., :512] = codes.reshape(*lead, 512)
    rows[..., 512:544] = scale.contiguous().view(torch.uint8).reshape(*lead, 32)
    rows[..., 544:] = x[..., 512:].to(torch.bfloat16).contiguous().view(torch.uint8).reshape(*lead, 128)
    return rows


def _run(q2, raw, cmp, idx, pos, raw_pt, cmp_pt, cmp_lens, n_tok, tok_per_seq, topk, window, raw_len, cmp_len,
         raw_ptw, cmp_ptw, scale, check):
    return ops.sparse_mla_fwd(q2, raw, cmp, idx, pos, raw_pt, cmp_pt, cmp_lens, n_tok, tok_per_seq, topk, window,
                              raw_len, cmp_len, raw_ptw, cmp_ptw, scale, check)


def prefill(q: torch.Tensor, kv: torch.Tensor, kv_cmp: torch.Tensor, indices: torch.Tensor, *, window: int = 128,
            softmax_scale: float | None = None, q_offset: int = 0, q_pos: torch.Tensor | None = None,
            check: bool = False):
    """q bf16 [B,S,128,576]; kv uint8 [B,S_raw,672] raw latent rows (query s sits at
    position s + q_offset < S_raw, or at ``q_pos[b, s]`` when given -- an arbitrary subset of
    a sequence's queries, e.g. one rank's shard); kv_cmp uint8 [B,G,672]; indices int32
    [B,S,topk] -> (o bf16 [B,S,128,512], lse fp32 [B,128,S])."""
    require_cuda(q, kv, kv_cmp, indices)
    assert q.dtype == torch.bfloat16 and q.dim() == 4 and q.shape[2:] == (H, DQK), \
        f"q must be bf16 [B, S, {H}, {DQK}], got {q.dtype} {tuple(q.shape)}"
    B, S = q.shape[:2]
    assert kv.dtype == torch.uint8 and kv.dim() == 3 and kv.shape[0] == B and kv.shape[2] == ROW_BYTES
    assert kv_cmp.dtype == torch.uint8 and kv_cmp.dim() == 3 and kv_cmp.shape[0] == B and kv_cmp.shape[2] == ROW_BYTES
    assert indices.dim() == 3 and indices.shape[:2] == (B, S), f"indices must be [B, S, topk], got {tuple(indices.shape)}"
    assert isinstance(window, int) and window >= 1, f"window must be a positive int, got {window!r}"
    topk = indices.shape[2]
    idx = indices.to(torch.int32).contiguous()
    if q_pos is None:
        assert q_offset >= 0 and S + q_offset <= kv.shape[1], "every query position must have its raw KV row"
        pos = (torch.arange(S, device=q.device, dtype=torch.int32) + q_offset).repeat(B)
    else:
        assert q_pos.shape == (B, S), f"q_pos must be [B, S]={(B, S)}, got {tuple(q_pos.shape)}"
        pos = q_pos.to(device=q.device, dtype=torch.int32).contiguous().view(B * S)
        if check and S:
            assert 0 <= int(pos.min()) and int(pos.max()) < kv.shape[1], "every query position must have its raw KV row"
    cmp = kv_cmp if kv_cmp.shape[1] else kv  # never dereferenced when G == 0
    scale = softmax_scale if softmax_scale is not None else DQK**-0.5
    o, lse = _run(q.contiguous(), kv.contiguous(), cmp.contiguous(), idx, pos, None, None, None, B * S, S, topk,
                  window, kv.shape[1], kv_cmp.shape[1], 0, 0, float(scale), check)
    return o.view(B, S, H, DV), lse.view(B, S, H).permute(0, 2, 1).contiguous()


def decode(q: torch.Tensor, kv_pages: torch.Tensor, page_table: torch.Tensor, seq_lens: torch.Tensor,
           cmp_pages: torch.Tensor, cmp_page_table: torch.Tensor, cmp_lens: torch.Tensor, indices: torch.Tensor, *,
           window: int = 128, softmax_scale: float | None = None, check: bool = False):
    """One new token per sequence at position ``seq_lens[b] - 1``.

    q bf16 [B,128,576]; kv_pages uint8 [P,64,672] raw latent pages with page_table int32
    [B, max_pages]; cmp_pages uint8 [Pc,64,672] compressed pages with cmp_page_table
    [B, max_cmp_pages] and cmp_lens [B] valid compressed entries; indices int32 [B,topk]
    (compressed positions, -1 = empty) -> (o bf16 [B,128,512], lse fp32 [B,128])."""
    require_cuda(q, kv_pages, page_table, seq_lens, cmp_pages, cmp_page_table, cmp_lens, indices)
    assert q.dtype == torch.bfloat16 and q.dim() == 3 and q.shape[1:] == (H, DQK)
    B = q.shape[0]
    assert kv_pages.dtype == torch.uint8 and kv_pages.shape[1:] == (64, ROW_BYTES)
    assert cmp_pages.dtype == torch.uint8 and cmp_pages.shape[1:] == (64, ROW_BYTES)
    assert page_table.shape[0] == B and cmp_page_table.shape[0] == B and indices.shape[0] == B
    pos = (seq_lens.to(torch.int32) - 1).contiguous()
    topk = indices.shape[1]
    scale = softmax_scale if softmax_scale is not None else DQK**-0.5
    return _run(q.contiguous(), kv_pages.contiguous(), cmp_pages.contiguous(), indices.to(torch.int32).contiguous(),
                pos, page_table.to(torch.int32).contiguous(), cmp_page_table.to(torch.int32).contiguous(),
                cmp_lens.to(torch.int32).contiguous(), B, 1, topk, window, 0, 0, page_table.shape[1],
                cmp_page_table.shape[1], float(scale), check)


def pair_flops(pairs: int, heads: int = H) -> float:
    """Algorithmic FLOPs of `pairs` selected (query, key) pairs: 2 * heads * (576 + 512) each."""
    return 2.0 * heads * (DQK + DV) * float(pairs)
