"""Lightning indexer with mzoo's call signatures, on sm_100a kernels.

Drop-in for ``src/mzoo/layers/attn/indexer``:

- ``fwd(q, k, w, *, compress_ratio)`` -> fp32 [B,S,T] scores  (``indexer/fwd.py:112``)
- ``attn(q, k, w, *, compress_ratio, topk)`` -> int32 [B,S,topk] (``indexer/attn.py:67``)

Additive keyword arguments (defaults reproduce the reference):

- ``q_offset`` -- absolute position of query 0 (the model's ``position_ids``,
  ``archs/dsv4/modeling_deepseek_v41.py:555``); the reference kernel assumes 0.
- ``scales=(sq, sk)`` -- FP8 mode: ``q``/``k`` are ``torch.float8_e4m3fn`` codes with
  fp32 scales per (token, head) ``[B,S,Hi]`` and per key ``[B,T]``.
- ``softmax_scale`` -- the overall factor (default ``Di**-0.5`` in bf16 mode, 1 in fp8).
- ``q_pos`` -- int32 [B, S] absolute position per query (decode: ``seq_len - 1``);
  overrides ``q_offset``.
- ``k_page_table`` -- int32 [B, pages]: paged keys (a decode KV cache) -- ``k`` is then
  [P, 64, Di] (64 key rows per page, fp8 scales ``sk`` [P, 64]) and key t of batch b is
  row t % 64 of page ``k_page_table[b, t // 64]``; T = 64 * pages (keys past a sequence's
  visible count are never used, whatever its table holds there).

``attn`` returns, per query, the indices of the ``topk`` largest scores -- exact with
respect to the fp64 canonical score (see ``csrc/indexer.cu``), ties to the lower index --
in ascending order, ``-1`` padded where fewer keys are visible.  (The reference returns
``torch.topk(sorted=False)`` order; its tests compare sets.)
"""

import torch

from . import ops
from ._lib import require_cuda

KB_PARTS = 16
# relative bound on the fp32 tensor-core score error: |approx - exact| <= EPS * A_s * B_t
EPS = 2.0**-21


def _prep(q, k, w, scales, softmax_scale, k_page_table=None):
    require_cuda(q, k, w)
    fp8 = q.dtype == torch.float8_e4m3fn
    if fp8:
        assert k.dtype == torch.float8_e4m3fn, f"fp8 q needs fp8 k, got {k.dtype}"
        assert scales is not None, "fp8 inputs need scales=(sq [B,S,Hi], sk [B,T])"
        sq, sk = (s.float().contiguous() for s in scales)
    else:
        assert q.dtype == k.dtype == torch.bfloat16, f"q/k must be bf16, got {q.dtype}/{k.dtype}"
        assert scales is None, "scales are for fp8 inputs only"
        sq = sk = None
    B, S, Hi, Di = q.shape
    if k_page_table is None:
        assert k.dim() == 3 and k.shape[0] == B and k.shape[2] == Di, f"k must be [B, T, {Di}], got {tuple(k.shape)}"
    else:
        assert k.dim() == 3 and k.shape[1] == 64 and k.shape[2] == Di, \
            f"paged k must be [pages, 64, {Di}], got {tuple(k.shape)}"
        assert k_page_table.dim() == 2 and k_page_table.shape[0] == B, \
            f"k_page_table must be [B, pages], got {tuple(k_page_table.shape)}"
    assert w.shape == (B, S, Hi), f"w must be [B, S, Hi]={(B, S, Hi)}, got {tuple(w.shape)}"
    if sq is not None:
        assert sq.shape == (B, S, Hi) and sk.shape == k.shape[:2], "scales must be [B,S,Hi] and k's leading dims"
    w = w.float().contiguous()
    q, k = q.contiguous(), k.contiguous()
    if Hi % 16:  # the kernel tiles heads by 16: zero-weight heads contribute exactly 0
        pad = 16 - Hi % 16
        q = torch.cat([q, q.new_zeros(B, S, pad, Di)], dim=2)
        w = torch.cat([w, w.new_zeros(B, S, pad)], dim=2).contiguous()
        if sq is not None:
            sq = torch.cat([sq, sq.new_ones(B, S, pad)], dim=2).contiguous()
    scale = softmax_scale if softmax_scale is not None else (1.0 if fp8 else Di**-0.5)
    dt = 3 if fp8 else 1
    return q, k, w, sq, sk, float(scale), dt


def _scores(q, k, w, sq, sk, ratio, q_offset, scale, dt, write_tail, check, q_pos=None, k_pt=None):
    return ops.indexer_scores(q, k, w, sq, sk, q_pos, k_pt, ratio, q_offset, scale, dt, write_tail, check)


def _page_table(k_page_table, device):
    if k_page_table is None:
        return None
    return k_page_table.to(device=device, dtype=torch.int32).contiguous()


def _positions(q_pos, B, S, device):
    if q_pos is None:
        return None
    q_pos = q_pos.to(device=device, dtype=torch.int32).contiguous()
    assert q_pos.shape == (B, S), f"q_pos must be [B, S]={(B, S)}, got {tuple(q_pos.shape)}"
    return q_pos


def fwd(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, *, compress_ratio: int, q_offset: int = 0,
        scales=None, softmax_scale: float | None = None, q_pos: torch.Tensor | None = None,
        k_page_table: torch.Tensor | None = None, check: bool = False) -> torch.Tensor:
    """Lightning-indexer score matrix (``indexer/fwd.py:112``): q bf16 [B,S,Hi,Di], k bf16
    [B,T,Di], w fp32 [B,S,Hi] (already scaled by Hi**-0.5) -> fp32 [B,S,T], ``-inf`` where
    ``t >= (q_offset + s + 1) // compress_ratio``."""
    assert compress_ratio >= 1, f"compress_ratio must be >= 1, got {compress_ratio}"
    q, k, w, sq, sk, scale, dt = _prep(q, k, w, scales, softmax_scale, k_page_table)
    B, S = q.shape[:2]
    kpt = _page_table(k_page_table, q.device)
    if (k.shape[1] if kpt is None else kpt.shape[1]) == 0:
        return q.new_empty((B, S, 0), dtype=torch.float32)
    return _scores(q, k, w, sq, sk, compress_ratio, q_offset, scale, dt, True, check, _positions(q_pos, B, S, q.device),
                   kpt)


def attn(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, *, compress_ratio: int, topk: int, q_offset: int = 0,
         scales=None, softmax_scale: float | None = None, q_pos: torch.Tensor | None = None,
         k_page_table: torch.Tensor | None = None, check: bool = False) -> torch.Tensor:
    """``indexer/attn.py:67``: -> ``Indices`` int32 [B,S,topk] (``-1`` = empty slot)."""
    assert topk >= 0, f"topk must be >= 0, got {topk}"
    assert compress_ratio >= 1, f"compress_ratio must be >= 1, got {compress_ratio}"
    q, k, w, sq, sk, scale, dt = _prep(q, k, w, scales, softmax_scale, k_page_table)
    B, S, Hi, Di = q.shape
    kpt = _page_table(k_page_table, q.device)
    T = k.shape[1] if kpt is None else 64 * kpt.shape[1]
    if topk == 0 or T == 0:
        return torch.full((B, S, topk), -1, dtype=torch.int32, device=q.device)
    qp = _positions(q_pos, B, S, q.device)
    sc = _scores(q, k, w, sq, sk, compress_ratio, q_offset, scale, dt, False, check, qp, kpt)
    return ops.indexer_topk(sc, q, k, w, sq, sk, qp, kpt, compress_ratio, q_offset, scale, dt, topk, EPS, KB_PARTS,
                            check)


def bwd(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, dl: torch.Tensor, *, compress_ratio: int,
        q_offset: int = 0, softmax_scale: float | None = None, check: bool = False):
    """``indexer/bwd.py:104``: q bf16 [B,S,Hi,Di], k bf16 [B,T,Di], w fp32 [B,S,Hi], dl fp32
    [B,S,T] -> (dq bf16 [B,S,Hi,Di], dk bf16 [B,T,Di], dw fp32 [B,S,Hi]).  Entries of ``dl`` at
    group-causally masked positions are ignored, whatever they hold."""
    require_cuda(q, k, w, dl)
    assert q.dtype == k.dtype == torch.bfloat16, f"q/k must be bf16, got {q.dtype}/{k.dtype}"
    B, S, Hi, Di = q.shape
    T = k.shape[1]
    assert k.shape == (B, T, Di) and w.shape == (B, S, Hi), "shape mismatch"
    assert dl.shape == (B, S, T) and dl.dtype == torch.float32, \
        f"dl must be [B,S,T] fp32, got {tuple(dl.shape)} {dl.dtype}"
    assert T > 0, "bwd of an empty key axis is all zeros -- handle at the caller"
    assert Di in (64, 96, 128, 256), f"indexer backward supports index head dim 64 / 96 / 128 / 256, got {Di}"
    hp = 16
    while hp < Hi:
        hp *= 2
    assert hp <= (128 if Di == 256 else 256), f"indexer backward: {Hi} heads at Di={Di} not supported"
    qp, wp, kp = q.contiguous(), w.float().contiguous(), k.contiguous()
    Dk = 128 if Di == 96 else Di  # zero channels: same dot products, zero gradient channels
    if Dk != Di:
        qp = torch.nn.functional.pad(qp, (0, Dk - Di)).contiguous()
        kp = torch.nn.functional.pad(kp, (0, Dk - Di)).contiguous()
    if hp != Hi:  # pad heads to a power of two >= 16 with zero weights (their gradients are discarded)
        qp = torch.cat([qp, qp.new_zeros(B, S, hp - Hi, Dk)], dim=2).contiguous()
        wp = torch.cat([wp, wp.new_zeros(B, S, hp - Hi)], dim=2).contiguous()
    scale = softmax_scale if softmax_scale is not None else Di**-0.5
    dq, dk, dw = ops.indexer_bwd(qp, kp, wp, dl.contiguous(), compress_ratio, q_offset, float(scale), check)
    return dq[:, :, :Hi, :Di].contiguous(), dk[..., :Di].contiguous(), dw[:, :, :Hi].contiguous()


class _ScoresAutograd(torch.autograd.Function):
    """``indexer/attn.py:37-50``: fwd + bwd glued; saves only q, k, w."""

    @staticmethod
    def forward(ctx, q, k, w, compress_ratio):
        ctx.save_for_backward(q, k, w)
        ctx.compress_ratio = compress_ratio
        return fwd(q, k, w, compress_ratio=compress_ratio)

    @staticmethod
    def backward(ctx, dl):
        q, k, w = ctx.saved_tensors
        dq, dk, dw = bwd(q, k, w, dl.contiguous().float(), compress_ratio=ctx.compress_ratio)
        return dq, dk, dw, None


def scores(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, *, compress_ratio: int,
           fake_quant_fp4: bool = False) -> torch.Tensor:
    """``indexer/attn.py:53``: differentiable ``fwd``.  ``fake_quant_fp4=True`` round-trips q/k
    through the fp4 block-32 quantiser with a straight-through gradient first
    (``indexer/attn.py:29-34``)."""
    if fake_quant_fp4:
        from .quant import fake_quant_fp4_ste
        q, k = fake_quant_fp4_ste(q, 32), fake_quant_fp4_ste(k, 32)
    return _ScoresAutograd.apply(q, k, w, compress_ratio)


def quantize_fp8(x: torch.Tensor, dim_tile: int | None = None):
    """Absmax e4m3 quantisation of indexer inputs: per row of the last
    dim (or per ``dim_tile`` elements), ``scale = amax / 448`` -> (codes, fp32 scales)."""
    xf = x.float()
    n = xf.shape[-1]
    tile = dim_tile or n
    blocks = xf.view(*xf.shape[:-1], n // tile, tile)
    amax = blocks.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = (blocks / scale.unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(x.shape)
    return codes, (scale.squeeze(-1) if dim_tile is None else scale)
