"""576/512 latent sparse attention oracle (numpy) -- test infrastructure, not the product.

Restates ``golden_ref._attend`` (golden_ref.py:83-100) for the shared-latent MQA with a
sliding window of raw tokens plus gathered compressed entries (``golden(level="sparse")``,
golden_ref.py:149-168), generalised to the DeepSeek-V4.1 latent layout BASELINE configs 3
and 4 use: K = the 576-dim latent (512 no-rope + 64 rope), V = its first 512 channels,
softmax scale ``576**-0.5`` unless given.

KV rows are stored as 672 bytes (the format ``mzoo_b200.sparse_mla`` reads):
``[0, 512)`` e4m3 codes of the no-rope part, ``[512, 544)`` 8 fp32 scales (one per
64-element tile, dequant = code * scale), ``[544, 672)`` 64 bf16 rope values.

Semantics (reference contract): a window of ``window`` raw tokens ending at the query's
position, itself included (``golden_ref.py:13-16``); compressed entries exactly as listed
in ``indices`` (-1 = empty slot, duplicates counted twice like the reference kernels,
``csa2_attn/bwd_dq.py:33-37``); one softmax over both; lse in natural log.
"""

import numpy as np

from .quant import FP8_MAX, bf16_to_f32, e4m3_round, f32_to_bf16

ROW_BYTES = 672
NOPE, ROPE, DQK, DV = 512, 64, 576, 512


def e4m3_codes(v: np.ndarray) -> np.ndarray:
    """float32 values on the e4m3 grid -> uint8 codes (sign | exp4 | man3)."""
    v = np.asarray(v, np.float32)
    a = np.abs(v).astype(np.float64)
    sign = np.signbit(v).astype(np.uint8) << 7
    codes = np.zeros(v.shape, np.uint8)
    sub = a < 2.0**-6
    codes[sub] = np.rint(a[sub] / 2.0**-9).astype(np.uint8)
    nrm = ~sub
    e = np.floor(np.log2(np.where(nrm, a, 1.0))).astype(np.int64)
    man = np.rint(a / np.exp2(e - 3)).astype(np.int64) - 8
    codes[nrm] = ((e[nrm] + 7) << 3 | man[nrm]).astype(np.uint8)
    return codes | sign


def e4m3_values(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    v = np.where(e == 0, m * 2.0**-9, (8 + m) * np.exp2(e - 10.0))
    return (s * v).astype(np.float32)


def pack_rows(kv: np.ndarray) -> np.ndarray:
    """[..., 576] float -> [..., 672] uint8 rows (absmax/448 scale per 64-tile, RTNE e4m3)."""
    kv = np.asarray(kv, np.float32)
    lead = kv.shape[:-1]
    nope = kv[..., :NOPE].reshape(*lead, 8, 64)
    amax = np.abs(nope).max(-1)
    scale = np.where(amax > 0, amax / FP8_MAX, np.float32(1.0)).astype(np.float32)
    q = np.clip((nope / scale[..., None]).astype(np.float32), -448, 448)
    codes = e4m3_codes(e4m3_round(q)).reshape(*lead, NOPE)
    rope = f32_to_bf16(kv[..., NOPE:])
    out = np.empty((*lead, ROW_BYTES), np.uint8)
    out[..., :NOPE] = codes
    out[..., NOPE:NOPE + 32] = scale.astype(np.float32).view(np.uint8).reshape(*lead, 32)
    out[..., NOPE + 32:] = rope.view(np.uint8).reshape(*lead, 128)
    return out


def unpack_rows(rows: np.ndarray) -> np.ndarray:
    """[..., 672] uint8 -> [..., 576] float32 (nope = code * scale in fp32, rope = bf16)."""
    rows = np.ascontiguousarray(rows, np.uint8)
    lead = rows.shape[:-1]
    vals = e4m3_values(rows[..., :NOPE]).reshape(*lead, 8, 64)
    scale = rows[..., NOPE:NOPE + 32].copy().view(np.float32).reshape(*lead, 8)
    nope = (vals * scale[..., None]).astype(np.float32).reshape(*lead, NOPE)
    rope = bf16_to_f32(rows[..., NOPE + 32:].copy().view(np.uint16).reshape(*lead, ROPE))
    return np.concatenate([nope, rope], -1)


def attend_rows(q: np.ndarray, keys: np.ndarray, scale: float) -> tuple:
    """One token: q [H, 576], keys [n, 576] (already gathered, duplicates kept) ->
    (o [H, 512], lse [H]) in float64."""
    q = np.asarray(q, np.float64)
    k = np.asarray(keys, np.float64)
    logits = (q @ k.T) * scale
    m = logits.max(-1, keepdims=True)
    p = np.exp(logits - m)
    l = p.sum(-1, keepdims=True)
    o = (p @ k[:, :DV]) / l
    return o, (m + np.log(l))[:, 0]


def token_keys(raw: np.ndarray, cmp: np.ndarray, idx_row: np.ndarray, pos: int, window: int) -> np.ndarray:
    """Dequantised key rows of one query: the window [pos-window+1, pos] of ``raw`` then the
    valid entries of ``idx_row`` in ``cmp`` ([n, 576] float32)."""
    lo = max(0, pos - window + 1)
    g = cmp.shape[0]
    sel = [int(i) for i in idx_row if 0 <= i < g]
    rows = [raw[lo:pos + 1]]
    if sel:
        rows.append(cmp[sel])
    return np.concatenate(rows, 0)


def sparse_prefill(q: np.ndarray, raw_rows: np.ndarray, cmp_rows: np.ndarray, idx: np.ndarray, window: int,
                   scale: float | None = None, tokens=None, q_offset: int = 0) -> tuple:
    """q [B,S,H,576] (bf16 values as float), raw_rows [B,S,672], cmp_rows [B,G,672],
    idx [B,S,topk] -> (o [B,S,H,512], lse [B,H,S]) float64 for the listed (b, s) tokens
    (all if ``tokens`` is None; others are NaN).  Query s sits at position ``s + q_offset``
    of ``raw_rows`` (raw_rows covers positions 0..S+q_offset-1 then)."""
    B, S, H, _ = q.shape
    scale = DQK**-0.5 if scale is None else scale
    raw = unpack_rows(raw_rows)
    cmp = unpack_rows(cmp_rows)
    o = np.full((B, S, H, DV), np.nan)
    lse = np.full((B, H, S), np.nan)
    todo = tokens if tokens is not None else [(b, s) for b in range(B) for s in range(S)]
    for b, s in todo:
        keys = token_keys(raw[b], cmp[b], idx[b, s], s + q_offset, window)
        o[b, s], lse[b, :, s] = attend_rows(q[b, s], keys, scale)
    return o, lse


def paged_rows(pages: np.ndarray, page_table: np.ndarray, b: int, positions) -> np.ndarray:
    """Rows of sequence b at token positions, through a page table of 64-token pages."""
    positions = np.asarray(positions, np.int64)
    return pages[page_table[b, positions // 64], positions % 64]


def sparse_decode(q: np.ndarray, raw_pages: np.ndarray, raw_pt: np.ndarray, seq_lens: np.ndarray,
                  cmp_pages: np.ndarray, cmp_pt: np.ndarray, cmp_lens: np.ndarray, idx: np.ndarray, window: int,
                  scale: float | None = None, seqs=None) -> tuple:
    """One new token per sequence at position L-1: window of raw positions [L-window, L-1]
    plus the compressed entries idx[b] (< cmp_lens[b]), all read through page tables.
    q [B,H,576] -> (o [B,H,512], lse [B,H]) float64."""
    B, H, _ = q.shape
    scale = DQK**-0.5 if scale is None else scale
    o = np.full((B, H, DV), np.nan)
    lse = np.full((B, H), np.nan)
    for b in (range(B) if seqs is None else seqs):
        L = int(seq_lens[b])
        lo = max(0, L - window)
        rows = [paged_rows(raw_pages, raw_pt, b, np.arange(lo, L))]
        sel = [int(i) for i in idx[b] if 0 <= i < int(cmp_lens[b])]
        if sel:
            rows.append(paged_rows(cmp_pages, cmp_pt, b, sel))
        keys = unpack_rows(np.concatenate(rows, 0))
        o[b], lse[b] = attend_rows(q[b], keys, scale)
    return o, lse
