"""``torch.library`` custom ops ``mzb::*`` -- the only place Python calls the C ABI.

Each op checks device / dtype / contiguity on the host, allocates its outputs with
torch (the library never allocates), passes raw pointers and the current stream to
``libmzb200.so`` and raises on a non-zero status.  Every op has a fake (meta)
implementation so it traces under ``torch.compile`` / ``FakeTensor`` without running.
"""

import torch

from . import _lib
from ._lib import call, ptr, require_cuda, stream_ptr


def _rows_n(x: torch.Tensor) -> tuple:
    n = x.shape[-1] if x.dim() else 1
    return (x.numel() // n if n else 0), n


# ----------------------------------------------------------------------------- fake quant

@torch.library.custom_op("mzb::fq_fp4", mutates_args=())
def fq_fp4(x: torch.Tensor, block_size: int, rule: int) -> torch.Tensor:
    require_cuda(x)
    assert x.dtype in _lib.DTYPE_CODE, f"fake quant supports fp32/bf16/fp16, got {x.dtype}"
    x = x.contiguous()
    y = torch.empty_like(x)
    rows, n = _rows_n(x)
    call("mzb_fq_fp4", ptr(x), ptr(y), rows, n, _lib.DTYPE_CODE[x.dtype], block_size, rule, stream_ptr(x.device))
    return y


@fq_fp4.register_fake
def _(x, block_size, rule):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("mzb::fq_fp8", mutates_args=())
def fq_fp8(x: torch.Tensor, block_size: int, rule: int) -> torch.Tensor:
    require_cuda(x)
    assert x.dtype in _lib.DTYPE_CODE, f"fake quant supports fp32/bf16/fp16, got {x.dtype}"
    x = x.contiguous()
    y = torch.empty_like(x)
    rows, n = _rows_n(x)
    call("mzb_fq_fp8", ptr(x), ptr(y), rows, n, _lib.DTYPE_CODE[x.dtype], block_size, rule, stream_ptr(x.device))
    return y


@fq_fp8.register_fake
def _(x, block_size, rule):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


# Per-device persistent error words.  Kernels only ever set their error word (on a failure:
# a bounded wait that gave up, a top-k error band too wide), never clear it, so one word per
# device keeps the first failure of every launch made with check=False until
# ``check_errors`` reads it.  Launches made with check=True get a fresh word that is read
# (a host synchronisation) right after the launch.
_ERR_WORDS: dict = {}


def _err(dev, check: bool) -> torch.Tensor:
    if check:
        return torch.zeros(1, dtype=torch.int32, device=dev)
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _ERR_WORDS.get(i)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", i))
        _ERR_WORDS[i] = w
    return w


def _raise_code(code: int, what: str) -> None:
    if code == _lib.MZB_ERR_BOUND:
        raise _lib.MzbError(f"{what}: error bound left too many top-k candidates")
    if code:
        raise _lib.MzbError(f"{what}: device error code {code} (a bounded device wait gave up)")


def _raise_on(err: torch.Tensor, what: str) -> None:
    _raise_code(int(err.item()), what)


def check_errors(device=None) -> None:
    """Raise ``MzbError`` if a kernel launched with ``check=False`` (the wrappers' default)
    on ``device`` (every device used so far when None) recorded a device-side failure since
    the last call; the word is cleared either way.  Reading it waits for the device's
    pending work, so call it where the caller synchronises anyway (end of a step)."""
    idx = list(_ERR_WORDS) if device is None else [torch.device(device).index or 0]
    first = 0
    for i in idx:
        w = _ERR_WORDS.get(i)
        if w is None:
            continue
        code = int(w.item())
        if code:
            w.zero_()
            first = first or code
    _raise_code(first, "deferred kernel check")


# ----------------------------------------------------------------------------- indexer

def _keys_T(k: torch.Tensor, k_pt: torch.Tensor | None) -> int:
    """Logical keys per batch: k [B,T,Di] dense, or 64 per page-table entry (k [P,64,Di])."""
    return k.shape[1] if k_pt is None else 64 * k_pt.shape[1]


def _pages(k: torch.Tensor, k_pt: torch.Tensor | None) -> tuple:
    return (ptr(k_pt), 0, 0) if k_pt is None else (ptr(k_pt), k_pt.shape[1], k.shape[0])


@torch.library.custom_op("mzb::indexer_scores", mutates_args=())
def indexer_scores(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, sq: torch.Tensor | None,
                   sk: torch.Tensor | None, q_pos: torch.Tensor | None, k_pt: torch.Tensor | None, ratio: int,
                   q_offset: int, scale: float, dtype: int, write_tail: bool, check: bool) -> torch.Tensor:
    """fp32 [B,S,T] scores of ``mzb_indexer_scores`` (q [B,S,Hi,Di] and k [B,T,Di] contiguous, or
    paged k [P,64,Di] with page table k_pt [B, pages] and T = 64 * pages)."""
    B, S, Hi, Di = q.shape
    T = _keys_T(k, k_pt)
    out = torch.empty(B, S, T, device=q.device, dtype=torch.float32)
    err = _err(q.device, check)
    call("mzb_indexer_scores", ptr(q), ptr(k), ptr(w), ptr(sq), ptr(sk), ptr(q_pos), ptr(out), B, S, T, Hi, Di, dtype,
         ratio, q_offset, scale, int(write_tail), *_pages(k, k_pt), ptr(err), stream_ptr(q.device))
    if check:
        _raise_on(err, "indexer scores")
    return out


@indexer_scores.register_fake
def _(q, k, w, sq, sk, q_pos, k_pt, ratio, q_offset, scale, dtype, write_tail, check):
    return q.new_empty((q.shape[0], q.shape[1], _keys_T(k, k_pt)), dtype=torch.float32)


@torch.library.custom_op("mzb::indexer_topk", mutates_args=())
def indexer_topk(scores: torch.Tensor, q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, sq: torch.Tensor | None,
                 sk: torch.Tensor | None, q_pos: torch.Tensor | None, k_pt: torch.Tensor | None, ratio: int,
                 q_offset: int, scale: float, dtype: int, topk: int, eps: float, kb_parts: int,
                 check: bool) -> torch.Tensor:
    """int32 [B,S,topk] exact top-k of ``mzb_indexer_topk`` (ascending, -1 padded)."""
    B, S, Hi, Di = q.shape
    T = _keys_T(k, k_pt)
    out = torch.empty(B, S, topk, dtype=torch.int32, device=q.device)
    kb = torch.empty(B * kb_parts + B * S, dtype=torch.float32, device=q.device)  # key and query bounds
    err = _err(q.device, check)
    call("mzb_indexer_topk", ptr(scores), ptr(q), ptr(k), ptr(w), ptr(sq), ptr(sk), ptr(q_pos), ptr(kb), ptr(out),
         B, S, T, Hi, Di, dtype, ratio, q_offset, scale, topk, eps, *_pages(k, k_pt), ptr(err), stream_ptr(q.device))
    if check:
        _raise_on(err, "indexer top-k")
    return out


@indexer_topk.register_fake
def _(scores, q, k, w, sq, sk, q_pos, k_pt, ratio, q_offset, scale, dtype, topk, eps, kb_parts, check):
    return q.new_empty((q.shape[0], q.shape[1], topk), dtype=torch.int32)


@torch.library.custom_op("mzb::indexer_bwd", mutates_args=())
def indexer_bwd(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, dl: torch.Tensor, ratio: int, q_offset: int,
                scale: float, check: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dq bf16, dk bf16, dw fp32) of ``mzb_indexer_bwd`` (heads already padded to 2^n >= 16)."""
    B, S, Hi, Di = q.shape
    T = k.shape[1]
    dq = torch.empty(B, S, Hi, Di, dtype=torch.bfloat16, device=q.device)
    dk = torch.empty(B, T, Di, dtype=torch.bfloat16, device=q.device)
    dw = torch.empty(B, S, Hi, dtype=torch.float32, device=q.device)
    err = _err(q.device, check)
    call("mzb_indexer_bwd", ptr(q), ptr(k), ptr(w), ptr(dl), ptr(dq), ptr(dk), ptr(dw), B, S, T, Hi, Di, ratio,
         q_offset, scale, ptr(err), stream_ptr(q.device))
    if check:
        _raise_on(err, "indexer backward")
    return dq, dk, dw


@indexer_bwd.register_fake
def _(q, k, w, dl, ratio, q_offset, scale, check):
    B, S, Hi, Di = q.shape
    return (q.new_empty((B, S, Hi, Di), dtype=torch.bfloat16), q.new_empty((B, k.shape[1], Di), dtype=torch.bfloat16),
            q.new_empty((B, S, Hi), dtype=torch.float32))


# ----------------------------------------------------------------------------- window / sparse attention

@torch.library.custom_op("mzb::attn_fwd", mutates_args=())
def attn_fwd(q: torch.Tensor, kv: torch.Tensor, v: torch.Tensor | None, main_kv: torch.Tensor | None,
             idx: torch.Tensor | None, sinks: torch.Tensor | None, window: int, scale: float,
             check: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(o bf16 [B,S,H,D], lse fp32 [B,S*H] token-major) of ``mzb_attn_fwd``."""
    B, S, H, D = q.shape
    dev = q.device
    o = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, S * H, dtype=torch.float32, device=dev)
    err = _err(dev, check)
    G = main_kv.shape[1] if main_kv is not None else 0
    topk = idx.shape[2] if idx is not None else 0
    call("mzb_attn_fwd", ptr(q), ptr(kv), ptr(v), ptr(main_kv), ptr(idx), ptr(sinks), ptr(o), ptr(lse), B, S, H, D,
         window, G, topk, scale, ptr(err), stream_ptr(dev))
    if check:
        _raise_on(err, "attention forward")
    return o, lse


@attn_fwd.register_fake
def _(q, kv, v, main_kv, idx, sinks, window, scale, check):
    B, S, H, D = q.shape
    return q.new_empty((B, S, H, D), dtype=torch.bfloat16), q.new_empty((B, S * H), dtype=torch.float32)


@torch.library.custom_op("mzb::attn_bwd", mutates_args=())
def attn_bwd(q: torch.Tensor, kv: torch.Tensor, v: torch.Tensor | None, main_kv: torch.Tensor | None,
             idx: torch.Tensor | None, o: torch.Tensor, lse_rows: torch.Tensor, do: torch.Tensor, window: int,
             scale: float, check: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dq, dk, dv, dmain fp32, delta) of ``mzb_attn_bwd``; ``lse_rows`` fp32 [B,S*H]
    token-major.  dv is empty when v is None (dk then holds dK + dV), dmain empty without
    gathered keys; delta = rowsum(dO * O) fp32 [B, S*H rounded up to 128]."""
    B, S, H, D = q.shape
    dev = q.device
    rpad = -(-S * H // 128) * 128
    dq = torch.empty_like(q)
    dk = torch.empty(B, S, 1, D, dtype=torch.bfloat16, device=dev)
    dv = torch.empty_like(dk) if v is not None else q.new_empty((0,), dtype=torch.bfloat16)
    G = main_kv.shape[1] if main_kv is not None else 0
    topk = idx.shape[2] if idx is not None else 0
    dmain = torch.zeros(B, G, D, dtype=torch.float32, device=dev) if G else q.new_empty((0,), dtype=torch.float32)
    delta = torch.empty(B, rpad, dtype=torch.float32, device=dev)
    lse2 = torch.empty(B, rpad, dtype=torch.float32, device=dev)
    err = _err(dev, check)
    splits = _lib.lib().mzb_attn_bwd_splits(B, S, H, window)
    part = torch.empty(splits * B * S * 2 * D, dtype=torch.float32, device=dev)
    call("mzb_attn_bwd", ptr(q), ptr(kv), ptr(v), ptr(main_kv), ptr(idx), ptr(o), ptr(lse_rows), ptr(do), ptr(dq),
         ptr(dk), ptr(dv if v is not None else None), ptr(dmain if G else None), ptr(delta), ptr(lse2), ptr(part), splits,
         B, S, H, D, window, G, topk, scale, ptr(err), stream_ptr(dev))
    if check:
        _raise_on(err, "attention backward")
    return dq, dk, dv, dmain, delta


@attn_bwd.register_fake
def _(q, kv, v, main_kv, idx, o, lse_rows, do, window, scale, check):
    B, S, H, D = q.shape
    rpad = -(-S * H // 128) * 128
    G = main_kv.shape[1] if main_kv is not None else 0
    dv = q.new_empty((B, S, 1, D) if v is not None else (0,), dtype=torch.bfloat16)
    dmain = q.new_empty((B, G, D) if G else (0,), dtype=torch.float32)
    return (q.new_empty(q.shape, dtype=torch.bfloat16), q.new_empty((B, S, 1, D), dtype=torch.bfloat16), dv, dmain,
            q.new_empty((B, rpad), dtype=torch.float32))


# ----------------------------------------------------------------------------- sparse latent MLA

@torch.library.custom_op("mzb::sparse_mla_fwd", mutates_args=())
def sparse_mla_fwd(q: torch.Tensor, kv_raw: torch.Tensor, kv_cmp: torch.Tensor, idx: torch.Tensor,
                   pos: torch.Tensor, raw_pt: torch.Tensor | None, cmp_pt: torch.Tensor | None,
                   cmp_lens: torch.Tensor | None, n_tok: int, tok_per_seq: int, topk: int, window: int, raw_len: int,
                   cmp_len: int, raw_ptw: int, cmp_ptw: int, scale: float,
                   check: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(o bf16 [n_tok,128,512], lse fp32 [n_tok,128]) of ``mzb_sparse_mla_fwd``."""
    dev = q.device
    o = torch.empty(n_tok, 128, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(n_tok, 128, dtype=torch.float32, device=dev)
    slots = torch.empty(max(n_tok, 1), dtype=torch.int32, device=dev)
    err = _err(dev, check)
    splits = _lib.lib().mzb_sparse_mla_splits(n_tok)
    part = torch.empty(splits * n_tok * 128 * 513, dtype=torch.float32, device=dev) if splits > 1 else None
    call("mzb_sparse_mla_fwd", ptr(q), ptr(kv_raw), ptr(kv_cmp), ptr(idx), ptr(pos), ptr(raw_pt), ptr(cmp_pt),
         ptr(cmp_lens), ptr(slots), ptr(o), ptr(lse), n_tok, tok_per_seq, topk, window, raw_len, cmp_len, raw_ptw,
         cmp_ptw, scale, splits, ptr(part), ptr(err), stream_ptr(dev))
    if check:
        _raise_on(err, "sparse_mla")
    return o, lse


@sparse_mla_fwd.register_fake
def _(q, kv_raw, kv_cmp, idx, pos, raw_pt, cmp_pt, cmp_lens, n_tok, tok_per_seq, topk, window, raw_len, cmp_len,
      raw_ptw, cmp_ptw, scale, check):
    return q.new_empty((n_tok, 128, 512), dtype=torch.bfloat16), q.new_empty((n_tok, 128), dtype=torch.float32)


# ----------------------------------------------------------------------------- two-level indexer selection

@torch.library.custom_op("mzb::candidate_blocks", mutates_args=())
def candidate_blocks(logits: torch.Tensor, clens: torch.Tensor, topk_blocks: int, block_size: int,
                     want_mask: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(blocks int32 [rows, topk_blocks], mask uint8 [rows, T] or [0]) of ``mzb_candidate_blocks``
    (logits fp32 [rows, T], clens int32 [rows], both contiguous)."""
    rows, T = logits.shape
    dev = logits.device
    blocks = torch.empty(rows, topk_blocks, dtype=torch.int32, device=dev)
    mask = torch.empty((rows, T) if want_mask else (0,), dtype=torch.uint8, device=dev)
    call("mzb_candidate_blocks", ptr(logits), ptr(clens), ptr(blocks), ptr(mask) if want_mask else None, rows, T,
         block_size, topk_blocks, stream_ptr(dev))
    return blocks, mask


@candidate_blocks.register_fake
def _(logits, clens, topk_blocks, block_size, want_mask):
    rows, T = logits.shape
    return (logits.new_empty((rows, topk_blocks), dtype=torch.int32),
            logits.new_empty((rows, T) if want_mask else (0,), dtype=torch.uint8))


@torch.library.custom_op("mzb::candidate_topk", mutates_args=())
def candidate_topk(scores: torch.Tensor, blocks: torch.Tensor | None, mask: torch.Tensor | None, block_size: int,
                   topk: int) -> torch.Tensor:
    """int32 [rows, topk] of ``mzb_candidate_topk`` (scores fp32 [rows, T]; candidates as a block
    list int32 [rows, nblk] or a uint8 mask [rows, T])."""
    rows, T = scores.shape
    out = torch.empty(rows, topk, dtype=torch.int32, device=scores.device)
    nblk = blocks.shape[1] if blocks is not None else 0
    call("mzb_candidate_topk", ptr(scores), ptr(blocks), ptr(mask), rows, T, block_size, nblk, topk, ptr(out),
         stream_ptr(scores.device))
    return out


@candidate_topk.register_fake
def _(scores, blocks, mask, block_size, topk):
    return scores.new_empty((scores.shape[0], topk), dtype=torch.int32)


# ----------------------------------------------------------------------------- compressor producer step

@torch.library.custom_op("mzb::compress", mutates_args=())
def compress(kv: torch.Tensor, gate: torch.Tensor | None, norm_w: torch.Tensor, cos: torch.Tensor | None,
             sin: torch.Tensor | None, ratio: int, rope_dim: int, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(latent bf16 [B,G,D], cache bf16 [B,G,D] or [0]) of ``mzb_compress`` (kv / gate fp32
    [B, G*ratio, D] contiguous; cos / sin fp32 [B, G, rope_dim/2] or None: no cache entry)."""
    B, N, D = kv.shape
    G = N // ratio
    dev = kv.device
    latent = torch.empty(B, G, D, dtype=torch.bfloat16, device=dev)
    want = cos is not None
    cache = torch.empty((B, G, D) if want else (0,), dtype=torch.bfloat16, device=dev)
    call("mzb_compress", ptr(kv), ptr(gate), ptr(norm_w), ptr(cos), ptr(sin), ptr(latent), ptr(cache) if want else None,
         B, G, ratio, D, rope_dim, eps, stream_ptr(dev))
    return latent, cache


@compress.register_fake
def _(kv, gate, norm_w, cos, sin, ratio, rope_dim, eps):
    B, N, D = kv.shape
    G = N // ratio
    return (kv.new_empty((B, G, D), dtype=torch.bfloat16),
            kv.new_empty((B, G, D) if cos is not None else (0,), dtype=torch.bfloat16))


# ----------------------------------------------------------------------------- RMSNorm + RoPE prologue

@torch.library.custom_op("mzb::norm_rope_fwd", mutates_args=())
def norm_rope_fwd(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor | None, sin: torch.Tensor | None,
                  heads: int, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(out bf16 like x, rstd fp32 [rows]) of ``mzb_norm_rope_fwd``: x bf16 [rows, D] contiguous,
    w bf16 [D], cos / sin fp32 [rows / heads, rope_dim / 2] contiguous (None: no rope)."""
    rows, D = x.shape
    out = torch.empty_like(x)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    rd = 0 if cos is None else 2 * cos.shape[-1]
    call("mzb_norm_rope_fwd", ptr(x), ptr(w), ptr(cos), ptr(sin), ptr(out), ptr(rstd), rows, heads, D, rd, eps,
         stream_ptr(x.device))
    return out, rstd


@norm_rope_fwd.register_fake
def _(x, w, cos, sin, heads, eps):
    return torch.empty_like(x), x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("mzb::norm_rope_bwd", mutates_args=())
def norm_rope_bwd(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor | None, sin: torch.Tensor | None,
                  rstd: torch.Tensor, dy: torch.Tensor, heads: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(dx bf16 like x, dw fp32 [D]) of ``mzb_norm_rope_bwd`` (dw summed over rows in a fixed
    order through a [parts, D] fp32 workspace)."""
    rows, D = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(D, dtype=torch.float32, device=x.device)
    parts = _lib.lib().mzb_norm_rope_bwd_parts(rows, D)
    part = torch.empty(parts * D, dtype=torch.float32, device=x.device)
    rd = 0 if cos is None else 2 * cos.shape[-1]
    call("mzb_norm_rope_bwd", ptr(x), ptr(dy), ptr(w), ptr(rstd), ptr(cos), ptr(sin), ptr(dx), ptr(part), ptr(dw), rows,
         heads, D, rd, parts, stream_ptr(x.device))
    return dx, dw


@norm_rope_bwd.register_fake
def _(x, w, cos, sin, rstd, dy, heads):
    return torch.empty_like(x), x.new_empty((x.shape[1],), dtype=torch.float32)


# ----------------------------------------------------------------------------- self-test

def selftest_bounded_wait(device, limit_ns: int, scope: int, check: bool) -> int:
    """Launch ``mzb_selftest_bounded_wait``: a wait that nothing satisfies runs out after
    ``limit_ns`` and records its site code.  check=True returns the code of a fresh error
    word (synchronising); check=False records it in the device's persistent word (read by
    ``check_errors``) and returns 0."""
    dev = torch.device(device)
    err = _err(dev, check)
    call("mzb_selftest_bounded_wait", int(limit_ns), int(scope), ptr(err), stream_ptr(dev))
    return int(err.item()) if check else 0


# ----------------------------------------------------------------------------- KV cache formats

@torch.library.custom_op("mzb::kv_pack", mutates_args=())
def kv_pack(x: torch.Tensor, fmt: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``mzb_kv_pack_fp8`` (fmt 8: e4m3 codes [rows, D] + ue8m0 bytes [rows, D/32]) or
    ``mzb_kv_pack_fp4`` (fmt 4: packed e2m1 [rows, D/2] + e4m3 bytes [rows, D/16]) of a
    contiguous bf16 [rows, D]."""
    require_cuda(x)
    rows, D = x.shape
    if fmt == 8:
        codes = torch.empty(rows, D, dtype=torch.uint8, device=x.device)
        scales = torch.empty(rows, D // 32, dtype=torch.uint8, device=x.device)
        call("mzb_kv_pack_fp8", ptr(x), ptr(codes), ptr(scales), rows, D, stream_ptr(x.device))
    else:
        codes = torch.empty(rows, D // 2, dtype=torch.uint8, device=x.device)
        scales = torch.empty(rows, D // 16, dtype=torch.uint8, device=x.device)
        call("mzb_kv_pack_fp4", ptr(x), ptr(codes), ptr(scales), rows, D, stream_ptr(x.device))
    return codes, scales


@kv_pack.register_fake
def _(x, fmt):
    rows, D = x.shape
    if fmt == 8:
        return x.new_empty((rows, D), dtype=torch.uint8), x.new_empty((rows, D // 32), dtype=torch.uint8)
    return x.new_empty((rows, D // 2), dtype=torch.uint8), x.new_empty((rows, D // 16), dtype=torch.uint8)


@torch.library.custom_op("mzb::kv_unpack", mutates_args=())
def kv_unpack(codes: torch.Tensor, scales: torch.Tensor, D: int, fmt: int) -> torch.Tensor:
    """bf16 [rows, D] of ``mzb_kv_unpack_fp8`` / ``mzb_kv_unpack_fp4``."""
    require_cuda(codes, scales)
    rows = codes.shape[0]
    out = torch.empty(rows, D, dtype=torch.bfloat16, device=codes.device)
    name = "mzb_kv_unpack_fp8" if fmt == 8 else "mzb_kv_unpack_fp4"
    call(name, ptr(codes), ptr(scales), ptr(out), rows, D, stream_ptr(codes.device))
    return out


@kv_unpack.register_fake
def _(codes, scales, D, fmt):
    return codes.new_empty((codes.shape[0], D), dtype=torch.bfloat16)
