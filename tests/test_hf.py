"""The HF attention interface (``mzoo_b200.hf``) against the DeepSeek-V4.1 layer's eager
attention (``modeling_deepseek_v41.py:581-611``, restated in ``oracle/torch_ref.py``), on
the call the layer makes at ``:786``: q [B,H,S,D], kv [B,1,S+G,D] (K == V), the model's
window-causal mask with the indexer's block bias concatenated, the per-head sink.

CPU: registration, the block-bias -> indices conversion, and the glue with the kernel calls
replaced by a torch restatement (so the mapping of mask, window, sink and scale is what is
checked).  GPU: the real kernels, forward and gradients (q, kv, sinks), within 2e-2.
"""

import numpy as np
import pytest
import torch

from oracle import torch_ref as R

NEG = torch.finfo(torch.float32).min


class _Layer(torch.nn.Module):
    """The attributes of ``DeepseekV41Attention`` the interface reads."""

    def __init__(self, H, window, ratio, topk):
        super().__init__()
        self.attn_sink = torch.nn.Parameter(torch.randn(H))
        self.sliding_window = window
        self.compress_ratio = ratio
        self.config = type("Cfg", (), {"index_topk": topk})()


def _call(B=2, H=4, S=96, D=64, window=32, ratio=4, topk=8, seed=0, device="cpu"):
    """Inputs shaped like the layer's call: the raw mask uses finfo.min (HF's eager mask),
    the block bias 0 / -inf for a random causal selection of compressed groups."""
    g = torch.Generator().manual_seed(seed)
    G = S // ratio if ratio else 0
    q = torch.randn(B, H, S, D, generator=g)
    kv = torch.randn(B, 1, S + G, D, generator=g)
    t = torch.arange(S)
    vis = (t.view(-1, 1) - t.view(1, -1) < window) & (t.view(1, -1) <= t.view(-1, 1))
    raw = torch.zeros(S, S).masked_fill_(~vis, NEG).expand(B, 1, S, S)
    mask = raw
    if G:
        bias = torch.full((B, S, G), float("-inf"))
        for b in range(B):
            for s in range(S):
                nvis = (s + 1) // ratio
                if nvis:
                    pick = torch.randperm(nvis, generator=g)[:topk]
                    bias[b, s, pick] = 0.0
        mask = torch.cat([raw, bias.unsqueeze(1)], dim=-1)
    layer = _Layer(H, window, ratio, topk)
    return [x.to(device) for x in (q, kv, mask)] + [layer.to(device)]


def test_register_and_indices():
    hf = pytest.importorskip("mzoo_b200.hf")
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    name = hf.register()
    assert ALL_ATTENTION_FUNCTIONS.get_interface(name, None) is hf.attention_forward
    b = torch.full((1, 3, 6), float("-inf"))
    b[0, 0, [1, 4]] = 0
    b[0, 1, [0, 1, 2, 3, 5]] = 0
    got = hf.block_bias_to_indices(b, 4)
    assert got.tolist() == [[[1, 4, -1, -1], [0, 1, 2, 3], [-1, -1, -1, -1]]]


def test_glue_matches_eager_cpu(monkeypatch):
    """The kernels replaced by a float32 torch statement of what they compute: the glue's
    mapping must then reproduce the eager attention exactly (up to fp32 order)."""
    from mzoo_b200 import csa2_attn, hf, swa_attn

    def attend(q, kv, main, idx, window, sinks, scale):
        B, S, H, D = q.shape
        keys = kv[:, :, 0].float()
        logits = torch.einsum("bshd,btd->bhst", q.float(), keys) * scale
        t = torch.arange(S)
        vis = (t.view(-1, 1) - t.view(1, -1) < window) & (t.view(1, -1) <= t.view(-1, 1))
        logits = logits.masked_fill(~vis, float("-inf"))
        vals = keys
        if main is not None:
            m = main[:, :, 0].float()
            sel = torch.zeros(B, S, m.shape[1], dtype=torch.bool)
            bi, si, ki = torch.nonzero(idx >= 0, as_tuple=True)
            sel[bi, si, idx[bi, si, ki].long()] = True
            ml = torch.einsum("bshd,bgd->bhsg", q.float(), m) * scale
            logits = torch.cat([logits, ml.masked_fill(~sel.unsqueeze(1), float("-inf"))], -1)
            vals = torch.cat([keys, m], 1)
        logits = torch.cat([logits, sinks.float().view(1, H, 1, 1).expand(B, H, S, 1)], -1)
        p = torch.softmax(logits, -1)[..., :-1]
        return torch.einsum("bhst,btd->bshd", p, vals)

    monkeypatch.setattr(csa2_attn, "attn", lambda q, kv, main, idx, window, compress_ratio, causal, sinks,
                        softmax_scale: attend(q, kv, main, idx, window, sinks, softmax_scale))
    monkeypatch.setattr(swa_attn, "attn", lambda q, kv, window, causal, sinks, softmax_scale:
                        attend(q, kv, None, None, window, sinks, softmax_scale))
    for ratio in (4, 0):
        q, kv, mask, layer = _call(ratio=ratio)
        scale = q.shape[-1] ** -0.5
        got, _ = hf.attention_forward(layer, q, kv, kv, mask, scale, sliding_window=layer.sliding_window)
        ref = R.eager_sink_attention(q.bfloat16().float(), kv.bfloat16().float(), mask, layer.attn_sink, scale)
        assert float((got - ref).abs().max()) < 1e-4, ratio


def test_unsupported_calls_raise():
    from mzoo_b200 import hf
    q, kv, mask, layer = _call()
    with pytest.raises(NotImplementedError):
        hf.attention_forward(layer, q, kv, kv, mask, 0.1, dropout=0.1, sliding_window=32)
    with pytest.raises(NotImplementedError):  # a KV cache longer than... shorter than the queries
        hf.attention_forward(layer, q, kv[:, :, :10], kv[:, :, :10], mask[..., :10], 0.1, sliding_window=32)


@pytest.mark.gpu
@pytest.mark.parametrize("ratio", [4, 0])
def test_hf_attention_gpu(cuda, ratio):
    """Forward and gradients through the real kernels against the eager restatement."""
    from mzoo_b200 import hf
    q, kv, mask, layer = _call(B=2, H=8, S=256, D=128, window=64, ratio=ratio, topk=16, device=cuda)
    scale = q.shape[-1] ** -0.5
    qg = q.bfloat16().requires_grad_()
    kvg = kv.bfloat16().requires_grad_()
    o, _ = hf.attention_forward(layer, qg, kvg, kvg, mask, scale, sliding_window=layer.sliding_window)
    qr = q.bfloat16().float().requires_grad_()
    kvr = kv.bfloat16().float().requires_grad_()
    sinks_r = layer.attn_sink.detach().clone().requires_grad_()
    ref = R.eager_sink_attention(qr, kvr, mask, sinks_r, scale)
    assert float((o.detach().float() - ref.detach()).abs().max()) <= 2e-2
    do = torch.randn_like(ref)
    o.float().backward(do)
    ref.backward(do)
    for got, want, what in ((qg.grad, qr.grad, "dq"), (kvg.grad, kvr.grad, "dkv"),
                            (layer.attn_sink.grad, sinks_r.grad, "dsink")):
        err = float((got.float() - want).abs().max())
        tol = 2e-2 * max(1.0, float(want.abs().max()))
        assert err <= tol, (what, err, tol)
