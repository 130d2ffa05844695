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
    if not only or "candidates" in only:
        make_candidates()
    if not only or "compressor" in only:
        make_compressor()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
