"""The DeepSeek-V4.1 attention layer's HF attention interface, on this package's kernels.

``DeepseekV41Attention.forward`` (``modeling_deepseek_v41.py:786``) looks its attention up
with ``ALL_ATTENTION_FUNCTIONS.get_interface(config._attn_implementation,
eager_attention_forward)`` and calls it as

    fn(module, q [B,H,S,D], kv [B,1,T,D], kv, attention_mask, dropout=..., scaling=...,
       sliding_window=..., **kwargs) -> (attn_output [B,S,H,D], attn_weights)

where K == V is the shared latent, ``kv`` holds the window tokens' raw latents followed by
the group's compressed latents (T = S + G without a KV cache), and ``attention_mask`` is
the model's window-causal mask ``[B,1,S,S]`` with the indexer's per-query block bias
``[B,1,S,G]`` (0 for a selected compressed entry, -inf otherwise) concatenated
(``:766-780``).  The eager function (``:581-611``) adds the per-head ``module.attn_sink``
as one extra softmax logit that only grows the denominator.

``register()`` adds this module's ``attention_forward`` under the name ``"mzoo_b200"``;
a model configured with ``attn_implementation="mzoo_b200"`` then runs every attention
layer through ``csa2_attn`` (window + the selected compressed entries; ``swa_attn`` for a
layer without a compressed branch), with the sink, forward and backward.

Supported call: training / prefill without a KV cache (the first S rows of ``kv`` are the
query tokens' own latents), no attention dropout, head dims 64/96/128/256 (the reference's
csa2 / swa kernels stop at 256 as well).  Anything else raises ``NotImplementedError``:
there is no eager fallback here, so a model that should run on the kernels cannot
silently run off them.
"""

import torch

from . import csa2_attn, swa_attn

NAME = "mzoo_b200"


def block_bias_to_indices(bias: torch.Tensor, topk: int) -> torch.Tensor:
    """``[B,S,G]`` additive block bias (0 = selected, -inf = not) -> int32 ``[B,S,topk]``
    indices of the selected entries in ascending order, -1 padded (the ``indices`` argument
    of ``csa2_attn``).  Rows selecting more than ``topk`` entries keep the first ``topk``."""
    sel = bias == 0
    G = sel.shape[-1]
    if G == 0 or topk == 0:
        return torch.full((*sel.shape[:-1], topk), -1, dtype=torch.int32, device=bias.device)
    # a stable sort of "not selected" brings the selected entries to the front, in order
    order = torch.sort((~sel).to(torch.int8), dim=-1, stable=True).indices[..., :topk]
    if order.shape[-1] < topk:
        order = torch.nn.functional.pad(order, (0, topk - order.shape[-1]), value=0)
        keep = torch.gather(sel, -1, order) & (torch.arange(topk, device=bias.device) < G)
    else:
        keep = torch.gather(sel, -1, order)
    return torch.where(keep, order, torch.full_like(order, -1)).to(torch.int32)


def attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      attention_mask: torch.Tensor | None, scaling: float, dropout: float = 0.0,
                      sliding_window: int | None = None, **kwargs):
    """Drop-in for ``eager_attention_forward`` (``modeling_deepseek_v41.py:581``): returns
    ``(attn_output [B,S,H,D], None)``; the attention weights are not materialised."""
    if dropout:
        raise NotImplementedError("mzoo_b200 attention has no attention dropout (got dropout=%r)" % dropout)
    if value is not key and not torch.equal(value, key):
        raise NotImplementedError("mzoo_b200 attention is shared-latent MQA: key and value must be the same tensor")
    B, H, S, D = query.shape
    if key.dim() != 4 or key.shape[0] != B or key.shape[1] != 1 or key.shape[3] != D:
        raise NotImplementedError(f"mzoo_b200 attention expects kv [B,1,T,D], got {tuple(key.shape)}")
    T = key.shape[2]
    if T < S:
        raise NotImplementedError(
            f"mzoo_b200 attention: kv holds {T} rows for {S} queries; with a KV cache (decode) use "
            "sparse_mla.decode or the eager interface")
    window = int(sliding_window if sliding_window is not None else getattr(module, "sliding_window", 0) or 0)
    if window < 1:
        raise NotImplementedError("mzoo_b200 attention needs the layer's sliding window")
    ratio = int(getattr(module, "compress_ratio", 0) or 0)
    G = T - S
    if G and not ratio:
        raise NotImplementedError("mzoo_b200 attention: compressed rows on a layer without compress_ratio")
    sink = getattr(module, "attn_sink", None)
    q = query.transpose(1, 2).to(torch.bfloat16)             # [B,S,H,D]
    kv = key[:, 0, :S].unsqueeze(2).to(torch.bfloat16)        # [B,S,1,D], the window's raw latents
    if G == 0:
        o = swa_attn.attn(q, kv, window=window, causal=True, sinks=sink, softmax_scale=float(scaling))
        return o.to(query.dtype), None
    if attention_mask is None or attention_mask.shape[-1] != T:
        raise NotImplementedError("mzoo_b200 attention needs the mask with the indexer's block bias")
    topk = int(getattr(getattr(module, "config", None), "index_topk", 0) or G)
    if attention_mask.dtype == torch.bool:
        raise NotImplementedError("mzoo_b200 attention expects the additive (eager) mask; register() sets it")
    bias = attention_mask[:, 0, :, S:]
    idx = block_bias_to_indices(bias, min(topk, G))
    main = key[:, 0, S:].unsqueeze(2).to(torch.bfloat16)      # [B,G,1,D]
    o = csa2_attn.attn(q, kv, main, idx, window=window, compress_ratio=ratio, causal=True, sinks=sink,
                       softmax_scale=float(scaling))
    return o.to(query.dtype), None


def register(name: str = NAME) -> str:
    """Add ``attention_forward`` to transformers' attention registry under ``name``
    (``ALL_ATTENTION_FUNCTIONS``, the table ``modeling_deepseek_v41.py:786`` reads), and the
    eager mask builder under the same name: the layer concatenates its additive block bias
    onto the model's mask (``:766-772``), which needs the additive form, not sdpa's booleans."""
    from transformers.masking_utils import AttentionMaskInterface, eager_mask
    from transformers.modeling_utils import AttentionInterface
    # class-level registration: the model's mask builders consult the global table
    AttentionInterface.register(name, attention_forward)
    AttentionMaskInterface.register(name, eager_mask)
    return name
