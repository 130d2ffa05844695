"""Generate the golden input/output vectors under ``tests/golden/`` by running the
reference (pmonad/mzoo) itself on the CPU.

Run in a container where the reference sources are importable, e.g.::

    MZOO_REF_SRC=<path to mzoo>/src python tests/golden/make_golden.py

It imports the reference's pure-PyTorch functions
(``mzoo.archs.owlet1.quant``, ``mzoo.layers.attn.golden_ref``) and writes small ``.npz``
fixtures.  Nothing at test time imports the reference: the fixtures are the pin.
bf16 tensors are stored as uint16 bit patterns.
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref():
    src = os.environ.get("MZOO_REF_SRC")
    if src:
        sys.path.insert(0, src)
    from mzoo.archs.owlet1 import quant  # noqa: E402
    from mzoo.layers.attn import golden_ref  # noqa: E402
    return quant, golden_ref


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def quant_inputs(seed: int) -> dict:
    """Random blocks plus hand-picked edge cases: ties of the e2m1 grid, exact
    thresholds, zeros, negative zero, tiny (subnormal) and large magnitudes."""
    g = torch.Generator().manual_seed(seed)
    cases = {}
    cases["randn"] = torch.randn(8, 4, 128, generator=g)
    cases["wide"] = torch.randn(4, 256, generator=g) * torch.logspace(-30, 30, 256).view(1, 256)
    # e2m1 ties: an amax of 6 makes the ue8m0 scale exactly 1, so q == x
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0,
                         -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0,
                         0.0, -0.0, 0.2499, 0.2501, 0.7499, 0.7501, 1.2501, 1.7499,
                         2.4999, 2.5001, 3.4999, 3.5001, 4.9999, 5.0001, 1e-30, -1e-30])
    cases["ties"] = ties.view(1, 32)
    cases["zeros"] = torch.zeros(2, 64)
    cases["tiny"] = torch.randn(2, 64, generator=g) * 1e-38
    cases["huge"] = torch.randn(2, 64, generator=g) * 1e30
    # fp8: values straddling e4m3 rounding points after a pow2 scale of 1 (amax 448)
    fp8 = torch.tensor([448.0, 240.0, 232.0, 248.0, 17.0, 19.0, 0.001953125, 0.0029296875,
                        0.0009765625, 0.015625, 0.0146484375, -0.013671875, 1.0625, 1.1875, -3.25, 0.0])
    cases["fp8pts"] = fp8.repeat(2).view(1, 32)
    cases["ragged"] = torch.randn(3, 40, generator=g)  # 40 % 32 != 0 -> returned unchanged
    return cases


def make_quant(quant) -> None:
    out = {}
    for name, x in quant_inputs(0).items():
        for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            xx = x.to(dt)
            out[f"{name}.{tag}.x"] = bits(xx)
            out[f"{name}.{tag}.fp4_32"] = bits(quant._fake_quant_fp4_block(xx, 32))
            out[f"{name}.{tag}.fp4_16e4m3"] = bits(quant._fake_quant_fp4_block(xx, 16, e4m3_scales=True))
            out[f"{name}.{tag}.fp8_32"] = bits(quant._fake_quant_fp8_block(xx, 32))
            out[f"{name}.{tag}.fp8_16"] = bits(quant._fake_quant_fp8_block(xx, 16))
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)


def make_attention(golden_ref) -> None:
    out = {}
    g = torch.Generator().manual_seed(1)
    # window level, fp32, with and without sinks (golden_ref.py:103-147)
    b, s, h, d = 1, 96, 4, 32
    q = torch.randn(b, s, h, d, generator=g)
    kv = torch.randn(b, s, 1, d, generator=g)
    sinks = torch.randn(h, generator=g)
    for w in (1, 16, 40, 200):
        o, lse = golden_ref.golden(q, kv, level="window", window=w)
        out[f"window{w}.o"], out[f"window{w}.lse"] = o.numpy(), lse.numpy()
    o, lse = golden_ref.golden(q, kv, level="window", window=16, sinks=sinks)
    out["window16sink.o"], out["window16sink.lse"] = o.numpy(), lse.numpy()
    out["q"], out["kv"], out["sinks"] = q.numpy(), kv.numpy(), sinks.numpy()
    # sparse level: main_kv + indices with -1 padding and a duplicate (golden dedups)
    gcount, topk, ratio = 20, 8, 4
    main = torch.randn(b, gcount, 1, d, generator=g)
    vis = (torch.arange(s) + 1) // ratio
    idx = torch.full((b, s, topk), -1, dtype=torch.int64)
    for t in range(s):
        n = int(min(vis[t].item(), gcount))
        perm = torch.randperm(n, generator=g)[:topk] if n else torch.zeros(0, dtype=torch.int64)
        idx[0, t, :len(perm)] = perm
    o, lse = golden_ref.golden(q, kv, level="sparse", window=16, main_kv=main,
                               compress_ratio=ratio, indices=idx)
    out["main"], out["idx"] = main.numpy(), idx.numpy()
    out["sparse.o"], out["sparse.lse"] = o.numpy(), lse.numpy()
    # gradients of the window level through autograd (dq, dkv, dsinks)
    qg, kvg, sg = q.clone().requires_grad_(), kv.clone().requires_grad_(), sinks.clone().requires_grad_()
    o, _ = golden_ref.golden(qg, kvg, level="window", window=16, sinks=sg)
    do = torch.randn(o.shape, generator=g)
    o.backward(do)
    out["bwd.do"], out["bwd.dq"], out["bwd.dkv"], out["bwd.dsinks"] = (
        do.numpy(), qg.grad.numpy(), kvg.grad.numpy(), sg.grad.numpy())
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)


def make_indexer(golden_ref) -> None:
    out = {}
    g = torch.Generator().manual_seed(2)
    b, s, hi, di, t, ratio = 2, 64, 8, 32, 20, 2
    q = torch.randn(b, s, hi, di, generator=g)
    k = torch.randn(b, t, di, generator=g)
    w = torch.randn(b, s, hi, generator=g) * hi**-0.5
    sc = golden_ref.indexer_scores(q, k, w, ratio)
    out["q"], out["k"], out["w"], out["scores"] = q.numpy(), k.numpy(), w.numpy(), sc.numpy()
    for topk in (4, 16, 25):
        out[f"topk{topk}"] = golden_ref.topk_indices(sc, topk).numpy()
    # gradients through the reference's differentiable scores (autograd of indexer_scores)
    qg, kg, wg = (x.clone().requires_grad_() for x in (q, k, w))
    sg = golden_ref.indexer_scores(qg, kg, wg, ratio)
    dl = torch.randn(sg.shape, generator=g)
    sg.backward(dl)
    out["bwd.dl"], out["bwd.dq"], out["bwd.dk"], out["bwd.dw"] = (dl.numpy(), qg.grad.numpy(), kg.grad.numpy(),
                                                                  wg.grad.numpy())
    np.savez_compressed(os.path.join(HERE, "indexer.npz"), **out)


def _fp8_absmax(x: torch.Tensor, tile: int):
    """Absmax e4m3 quantisation in torch (the synthetic inputs' rule): per ``tile`` elements
    of the last axis scale = amax / 448 (1 where amax is 0), codes = e4m3(x / scale) with
    torch's own float8_e4m3fn cast (round to nearest even).  -> (uint8 codes, fp32 scales)."""
    lead = x.shape[:-1]
    blk = x.float().reshape(*lead, x.shape[-1] // tile, tile)
    amax = blk.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = (blk / scale.unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn)
    return codes.view(torch.uint8).reshape(x.shape), scale


def _e4m3_dequant(codes: torch.Tensor, scale: torch.Tensor, tile: int) -> torch.Tensor:
    lead = codes.shape[:-1]
    vals = codes.view(torch.float8_e4m3fn).float().reshape(*lead, codes.shape[-1] // tile, tile)
    return (vals * scale.unsqueeze(-1)).reshape(codes.shape)


def _pack_latent(x: torch.Tensor) -> torch.Tensor:
    """[..., 576] fp32 -> [..., 672] uint8 latent rows: 512 e4m3 codes (absmax/448 per 64),
    the 8 fp32 scales, the 64 rope channels as bf16."""
    lead = x.shape[:-1]
    codes, scale = _fp8_absmax(x[..., :512], 64)
    rows = torch.empty(*lead, 672, dtype=torch.uint8)
    rows[..., :512] = codes
    rows[..., 512:544] = scale.contiguous().view(torch.uint8).reshape(*lead, 32)
    rows[..., 544:] = x[..., 512:].to(torch.bfloat16).contiguous().view(torch.uint8).reshape(*lead, 128)
    return rows


def _unpack_latent(rows: torch.Tensor) -> torch.Tensor:
    """[..., 672] uint8 -> [..., 576] fp32 (nope = code * tile scale, rope = bf16 value)."""
    lead = rows.shape[:-1]
    scale = rows[..., 512:544].contiguous().view(torch.float32).reshape(*lead, 8)
    nope = _e4m3_dequant(rows[..., :512].contiguous(), scale, 64)
    rope = rows[..., 544:].contiguous().view(torch.bfloat16).float().reshape(*lead, 64)
    return torch.cat([nope, rope], -1)


def _attend_rows(golden_ref, q_tok: torch.Tensor, keys: torch.Tensor):
    """The reference's ``_attend`` (golden_ref.py:83-100) for one query token over its
    gathered key rows: K = the 576-wide rows, V = their first 512 channels, scale
    576**-0.5 (``_attend`` scales by q's last dim), no mask, no sink, fp32."""
    q = q_tok.float().view(1, q_tok.shape[0], 1, 576)      # [B=1, H, S=1, D]
    k = keys.float().view(1, 1, keys.shape[0], 576)         # [B=1, Hk=1, T, D]
    o, lse = golden_ref._attend(q, k, k[..., :512], None, None, torch.float32)
    return o.view(q_tok.shape[0], 512), lse.view(q_tok.shape[0])


def make_mla(golden_ref) -> None:
    """576/512 FP8-latent sparse attention (BASELINE configs 3 and 4) through the
    reference's ``_attend`` on the rows each query gathers: the causal window of ``window``
    raw tokens ending at the query position, then the listed compressed entries in order
    (duplicates kept, ``-1`` and out-of-range entries dropped -- the reference kernels'
    rule, ``csa2_attn/fwd.py:1-16``, ``bwd_dq.py:33-37``).  The FP8 rows are packed and
    dequantised here with torch's own e4m3 cast, independently of the oracle.  Heads = 8:
    the oracle is head-generic (the kernels' 128 heads are covered by the GPU tests)."""
    out = {}
    g = torch.Generator().manual_seed(5)
    H = 8
    # prefill: S queries at positions q_offset..q_offset+S-1
    S, q_offset, G, topk, window = 16, 8, 14, 10, 6
    q = torch.randn(S, H, 576, generator=g).to(torch.bfloat16)
    kv = torch.randn(S + q_offset, 576, generator=g) * 1.5
    cmp = torch.randn(G, 576, generator=g)
    kv[3, :64] = 0.0  # an all-zero 64-channel tile (scale 1, all codes 0)
    raw_rows, cmp_rows = _pack_latent(kv), _pack_latent(cmp)
    raw_f, cmp_f = _unpack_latent(raw_rows), _unpack_latent(cmp_rows)
    idx = torch.full((S, topk), -1, dtype=torch.int32)
    for s in range(S):
        vis = min(G, (s + q_offset + 1) // 2)
        sel = torch.randperm(vis, generator=g)[:topk].sort().values if vis else torch.zeros(0, dtype=torch.int64)
        idx[s, :len(sel)] = sel.to(torch.int32)
        if s % 3 == 0 and len(sel) >= 2:
            idx[s, 1] = idx[s, 0]      # duplicate: counted twice
        if s % 4 == 1 and len(sel) >= 3:
            idx[s, 2] = G + 5          # out of range: empty slot
    o = torch.empty(S, H, 512)
    lse = torch.empty(H, S)
    for s in range(S):
        pos = s + q_offset
        sel = [int(i) for i in idx[s] if 0 <= int(i) < G]
        keys = torch.cat([raw_f[max(0, pos - window + 1):pos + 1], cmp_f[sel]], 0)
        o[s], lse[:, s] = _attend_rows(golden_ref, q[s], keys)
    out.update({"pre.q": bits(q), "pre.kv": kv.numpy(), "pre.cmp": cmp.numpy(), "pre.raw_rows": raw_rows.numpy(),
                "pre.cmp_rows": cmp_rows.numpy(), "pre.idx": idx.numpy(), "pre.o": o.numpy(), "pre.lse": lse.numpy(),
                "pre.params": np.array([q_offset, window], np.int64)})
    # paged decode: one token per sequence at position L-1, rows through 64-token page tables
    lens = torch.tensor([70, 200, 9], dtype=torch.int32)
    B, topk, window, ratio = 3, 12, 16, 4
    n_pages = int(((lens + 63) // 64).sum())
    clens = lens // ratio
    n_cpages = int(((clens + 63) // 64).sum())
    raw_pages = _pack_latent(torch.randn(n_pages, 64, 576, generator=g))
    cmp_pages = _pack_latent(torch.randn(n_cpages, 64, 576, generator=g))
    rperm, cperm = torch.randperm(n_pages, generator=g), torch.randperm(n_cpages, generator=g)
    pt = torch.zeros(B, 4, dtype=torch.int32)
    cpt = torch.zeros(B, 1, dtype=torch.int32)
    ro = co = 0
    for b in range(B):
        npg, ncp = int((lens[b] + 63) // 64), int((clens[b] + 63) // 64)
        pt[b, :npg] = rperm[ro:ro + npg].to(torch.int32)
        cpt[b, :ncp] = cperm[co:co + ncp].to(torch.int32)
        ro, co = ro + npg, co + ncp
    didx = torch.full((B, topk), -1, dtype=torch.int32)
    for b in range(B):
        sel = torch.randperm(int(clens[b]), generator=g)[:topk].sort().values
        didx[b, :len(sel)] = sel.to(torch.int32)
    didx[1, 3] = didx[1, 2]  # duplicate
    qd = torch.randn(B, H, 576, generator=g).to(torch.bfloat16)
    od = torch.empty(B, H, 512)
    lsed = torch.empty(B, H)
    for b in range(B):
        L = int(lens[b])
        pos = torch.arange(max(0, L - window), L)
        sel = torch.tensor([int(i) for i in didx[b] if 0 <= int(i) < int(clens[b])], dtype=torch.int64)
        rows = torch.cat([raw_pages[pt[b, pos // 64].long(), pos % 64], cmp_pages[cpt[b, sel // 64].long(), sel % 64]])
        od[b], lsed[b] = _attend_rows(golden_ref, qd[b], _unpack_latent(rows))
    out.update({"dec.q": bits(qd), "dec.raw_pages": raw_pages.numpy(), "dec.cmp_pages": cmp_pages.numpy(),
                "dec.pt": pt.numpy(), "dec.cpt": cpt.numpy(), "dec.lens": lens.numpy(), "dec.clens": clens.numpy(),
                "dec.idx": didx.numpy(), "dec.o": od.numpy(), "dec.lse": lsed.numpy(),
                "dec.params": np.array([window], np.int64)})
    np.savez_compressed(os.path.join(HERE, "mla.npz"), **out)


def make_indexer_fp8(golden_ref) -> None:
    """The FP8 indexer (BASELINE config 2's numerics) through the reference's
    ``indexer_scores`` / ``topk_indices`` (golden_ref.py:213-243): q quantised per
    (token, head) and k per token to e4m3 with absmax / 448 scales (torch's cast), the
    reference fed the dequantised values q * s_q and k * s_k.  The reference's score
    carries Di**-0.5 (the kernel's ``softmax_scale``) and no position offset."""
    out = {}
    g = torch.Generator().manual_seed(6)
    b, s, hi, di, t, ratio = 2, 48, 16, 64, 24, 2
    q = torch.randn(b, s, hi, di, generator=g)
    k = torch.randn(b, t, di, generator=g)
    w = torch.randn(b, s, hi, generator=g) / 8
    qc, sq = _fp8_absmax(q, di)
    kc, sk = _fp8_absmax(k, di)
    qd, kd = _e4m3_dequant(qc, sq, di), _e4m3_dequant(kc, sk, di)
    sc = golden_ref.indexer_scores(qd, kd, w, ratio)
    out.update({"q": q.numpy(), "k": k.numpy(), "w": w.numpy(), "q_codes": qc.numpy(), "k_codes": kc.numpy(),
                "sq": sq[..., 0].numpy(), "sk": sk[..., 0].numpy(), "scores": sc.numpy(),
                "params": np.array([ratio], np.int64)})
    for topk in (5, 12, 30):
        out[f"topk{topk}"] = golden_ref.topk_indices(sc, topk).numpy()
    np.savez_compressed(os.path.join(HERE, "indexer_fp8.npz"), **out)


def make_norm_rope() -> None:
    """The model's own RMSNorm + RoPE composition (``DeepseekV41RMSNorm`` and
    ``apply_rotary_pos_emb``, modeling_deepseek_v41.py:49-63 / :405-425; the
    ``qk_norm_rope_eager`` of layers/attn/norm_rope.py:37-44) on fp32 inputs with its
    autograd gradients, and on bf16 inputs (forward only), for q-shaped and kv-shaped
    tensors and non-power-of-two sizes."""
    from mzoo.archs.dsv4.modeling_deepseek_v41 import DeepseekV41RMSNorm, apply_rotary_pos_emb  # noqa: E402
    out = {}
    g = torch.Generator().manual_seed(7)
    cases = [(2, 33, 3, 64, 16), (1, 20, 1, 128, 64), (1, 7, 5, 96, 24), (1, 6, 2, 256, 64)]
    for c, (b, s, h, d, rd) in enumerate(cases):
        x = torch.randn(b, s, h, d, generator=g)
        w = torch.randn(d, generator=g)
        pos = torch.arange(s, dtype=torch.float32) + 3.0
        freqs = pos[:, None] / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
        cos = freqs.cos()[None].expand(b, -1, -1).contiguous()
        sin = freqs.sin()[None].expand(b, -1, -1).contiguous()
        dy = torch.randn(b, s, h, d, generator=g)
        key = f"c{c}."
        for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            xx, ww = x.to(dt).clone().requires_grad_(dt == torch.float32), w.to(dt).clone()
            ww.requires_grad_(dt == torch.float32)
            norm = DeepseekV41RMSNorm(d, eps=1e-6).to(dt)
            y = apply_rotary_pos_emb(torch.func.functional_call(norm, {"weight": ww}, (xx,)), cos, sin)
            out[key + tag + ".x"], out[key + tag + ".w"], out[key + tag + ".y"] = bits(xx.detach()), bits(ww.detach()), \
                bits(y.detach())
            if dt == torch.float32:
                y.backward(dy)
                out[key + "dy"], out[key + "dx"], out[key + "dw"] = dy.numpy(), xx.grad.numpy(), ww.grad.numpy()
        out[key + "cos"], out[key + "sin"] = cos.numpy(), sin.numpy()
    np.savez_compressed(os.path.join(HERE, "norm_rope.npz"), **out)


def make_candidates() -> None:
    """Level one through the reference's ``select_candidate_blocks``
    (archs/owlet1/indexer.py:14-41 = archs/dsv4/modeling_deepseek_v41.py:427-454); level two
    as written in ``DeepseekV41Indexer.forward`` (modeling_deepseek_v41.py:566-578):
    masked_fill(~candidates, -inf), topk(min(topk, T)), picks at -inf dropped."""
    from mzoo.archs.owlet1.indexer import select_candidate_blocks  # noqa: E402
    out = {}
    g = torch.Generator().manual_seed(3)
    # (rows, T, ratio, block_size, topk_blocks, topk, position offset)
    cases = [(48, 45, 4, 8, 3, 10, 0),      # T not a multiple of 8; few reachable blocks early on
             (40, 300, 2, 8, 16, 24, 100),  # more reachable blocks than topk_blocks
             (16, 37, 1, 4, 64, 5, 0),      # topk_blocks > number of blocks
             (24, 200, 1, 8, 5, 12, 150)]   # compress_len beyond T for the late rows: no pin
    for c, (rows, T, ratio, bs, tb, topk, off) in enumerate(cases):
        pos = off + torch.arange(rows) * max(1, (T * ratio) // rows)
        clen = ((pos + 1) // ratio).unsqueeze(-1)  # [rows, 1], the reference's trailing axis
        vis = torch.arange(T).view(1, -1) < clen
        logits = torch.where(vis, torch.randn(rows, T, generator=g), torch.tensor(float("-inf")))
        if c == 0:  # rows whose newest block also holds their best score
            for r in range(0, rows, 5):
                n = int(clen[r])
                if n > 0:
                    logits[r, n - 1] = 10.0
        mask = select_candidate_blocks(logits, clen, tb, bs)
        scores2 = torch.where(vis, torch.randn(rows, T, generator=g), torch.tensor(float("-inf")))
        masked = scores2.masked_fill(~mask, float("-inf"))
        top = masked.topk(min(topk, T), dim=-1, sorted=False)
        picks = torch.where(top.values > float("-inf"), top.indices, torch.full_like(top.indices, T))
        picks = picks.sort(dim=-1).values
        picks = torch.where(picks == T, torch.full_like(picks, -1), picks)  # -1 padding at the end
        key = f"c{c}."
        out[key + "logits"], out[key + "clen"] = logits.numpy(), clen.squeeze(-1).numpy().astype(np.int64)
        out[key + "mask"] = mask.numpy()
        out[key + "scores2"], out[key + "topk_idx"] = scores2.numpy(), picks.numpy().astype(np.int64)
        out[key + "params"] = np.array([bs, tb, topk], np.int64)
    np.savez_compressed(os.path.join(HERE, "candidates.npz"), **out)


def make_compressor() -> None:
    """The reference's own ``DeepseekV41Compressor`` (modeling_deepseek_v41.py:295-340, bf16
    module), ``apply_rotary_pos_emb`` (:405-425) and ``_fake_quant_fp4_block(..., 16,
    e4m3_scales=True)`` (:753) on seeded inputs; the fp32 projections kv / gate are stored as
    the kernel's inputs (the same F.linear calls the module makes)."""
    from types import SimpleNamespace  # noqa: E402

    import torch.nn.functional as F  # noqa: E402
    from mzoo.archs.dsv4.modeling_deepseek_v41 import (  # noqa: E402
        DeepseekV41Compressor, _fake_quant_fp4_block, apply_rotary_pos_emb)
    out = {}
    g = torch.Generator().manual_seed(4)
    # (batch, tokens, hidden, head_dim, rope_dim, ratio): tokens past the last full group dropped
    cases = [(2, 42, 256, 576, 64, 4), (1, 24, 128, 128, 32, 1), (2, 33, 192, 96, 16, 8)]
    for c, (b, s, hid, d, rd, ratio) in enumerate(cases):
        cfg = SimpleNamespace(compress_ratios=[ratio], head_dim=d, hidden_size=hid, rms_norm_eps=1e-6)
        m = DeepseekV41Compressor(cfg, 0)
        with torch.no_grad():
            m.wkv.weight.copy_(torch.randn(d, hid, generator=g) * hid**-0.5)
            if m.wgate is not None:
                m.wgate.weight.copy_(torch.randn(d, hid, generator=g) * hid**-0.5)
            m.norm.weight.copy_(1.0 + 0.25 * torch.randn(d, generator=g))
        m = m.to(torch.bfloat16)
        hs = torch.randn(b, s, hid, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            latent, _ = m(hs, None)
            usable = (s // ratio) * ratio
            if ratio > 1:
                kv = F.linear(hs.float(), m.wkv.weight.float())[:, :usable]
                gate = F.linear(hs.float(), m.wgate.weight.float())[:, :usable]
            else:  # no pooling: the projection in the model dtype
                kv, gate = m.wkv(hs).float(), None
            G = latent.shape[1]
            ang = torch.rand(b, G, rd // 2, generator=g) * 6.0
            cos, sin = ang.cos(), ang.sin()
            rotated = apply_rotary_pos_emb(latent, cos, sin)
            cache = _fake_quant_fp4_block(rotated, block_size=16, e4m3_scales=True)
        key = f"c{c}."
        out[key + "kv"] = kv.numpy()
        if gate is not None:
            out[key + "gate"] = gate.numpy()
        out[key + "norm_w"] = bits(m.norm.weight.detach())
        out[key + "cos"], out[key + "sin"] = cos.numpy(), sin.numpy()
        out[key + "latent"], out[key + "rotated"], out[key + "cache"] = bits(latent), bits(rotated), bits(cache)
        out[key + "params"] = np.array([ratio, rd], np.int64)
    np.savez_compressed(os.path.join(HERE, "compressor.npz"), **out)


def make_kvcache() -> None:
    """The model's two cache quantizers (modeling_deepseek_v41.py:359-402, :668-683):
    ``_fake_quant_fp8_block(x, 32)`` (window cache: e4m3, ue8m0 scale per 32 channels,
    amax clamped to 1e-4) and ``_fake_quant_fp4_block(x, 16, e4m3_scales=True)`` (main
    cache: e2m1, e4m3 scale per 16 channels, amax clamped to 6 * 2**-9), on bf16 rows with
    the edge cases the rules have: all-zero blocks (the clamp floors), exact e2m1 ties at
    0.25 / 0.75 / 1.25 / 1.75 / 2.5 / 3.5 / 5 times the scale, negative zeros and values
    at the clip limits.  Stores the dequantized outputs, and for fp4 the codes and e4m3
    scales the function forms on the way (its own ``_e2m1_codes`` / scale line)."""
    from mzoo.archs.dsv4 import modeling_deepseek_v41 as m  # noqa: E402
    g = torch.Generator().manual_seed(11)
    out = {}
    for c, (rows, d) in enumerate([(64, 128), (33, 64), (17, 256), (9, 96)]):
        x = torch.randn(rows, d, generator=g) * torch.exp2(torch.randint(-6, 6, (rows, 1), generator=g).float())
        x[0, :32] = 0.0                                   # zero blocks: the clamp floors
        x[1, :16] = -0.0
        ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0])
        x[2, :16] = ties                                  # amax 6 -> e4m3 scale 1: exact ties
        x[3, :32] = torch.linspace(-448.0, 448.0, 32)     # the e4m3 clip limits
        xb = x.to(torch.bfloat16)
        key = f"c{c}."
        out[key + "x"] = bits(xb)
        out[key + "fp8"] = bits(m._fake_quant_fp8_block(xb, 32))
        out[key + "fp4"] = bits(m._fake_quant_fp4_block(xb, 16, e4m3_scales=True))
        blocks = xb.float().view(rows, d // 16, 16)
        amax = blocks.abs().amax(-1)
        scale = (amax.clamp_min(6.0 * 2.0**-9) / m._FP4_MAX).to(torch.float8_e4m3fn)
        q = (blocks / scale.float().unsqueeze(-1)).clamp(-m._FP4_MAX, m._FP4_MAX)
        out[key + "fp4_codes"] = m._e2m1_codes(q).view(rows, d).numpy()
        out[key + "fp4_scales"] = scale.view(torch.uint8).numpy()
    np.savez_compressed(os.path.join(HERE, "kvcache.npz"), **out)


if __name__ == "__main__":
    torch.set_num_threads(1)
    quant, golden_ref = _ref()
    only = sys.argv[1:]
    if not only or "quant" in only:
        make_quant(quant)
    if not only or "attention" in only:
        make_attention(golden_ref)
    if not only or "indexer" in only:
        make_indexer(golden_ref)
    if not only or "mla" in only:
        make_mla(golden_ref)
    if not only or "indexer_fp8" in only:
        make_indexer_fp8(golden_ref)
    if not only or "norm_rope" in only:
        make_norm_rope()
    if not only or "candidates" in only:
        make_candidates()
    if not only or "compressor" in only:
        make_compressor()
    if not only or "kvcache" in only:
        make_kvcache()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
