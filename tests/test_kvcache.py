"""KV-cache formats (F2): the CPU restatement pinned to the model's own quantisers, the CUDA
packers bit-exact against it, and the attention over the packed caches equal to
``csa2_attn`` on the dequantised tensors (``tickets/0010-csa2-fp-cache.md``)."""

import os

import numpy as np
import pytest
import torch

from oracle import kvcache as K

HERE = os.path.dirname(os.path.abspath(__file__))


def _fixture():
    return np.load(os.path.join(HERE, "golden", "kvcache.npz"))


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def _cases():
    g = _fixture()
    return [(g[f"c{c}.x"], g[f"c{c}.fp8"], g[f"c{c}.fp4"], g[f"c{c}.fp4_codes"], g[f"c{c}.fp4_scales"])
            for c in range(4)]


def test_oracle_matches_model_quantisers():
    """The restatement's dequantised values are the model's, bit for bit; its fp4 codes and
    e4m3 scales are the ones the model's function forms."""
    for x, fp8, fp4, codes, scales in _cases():
        xb = _bf16(x)
        _, _, d8 = K.pack_window(xb)
        assert torch.equal(d8.view(torch.int16), _bf16(fp8).view(torch.int16))
        packed, sc, d4 = K.pack_main(xb)
        assert torch.equal(d4.view(torch.int16), _bf16(fp4).view(torch.int16))
        assert np.array_equal(sc.numpy(), scales)
        c = torch.from_numpy(codes)
        assert torch.equal(packed, c[:, 0::2] | (c[:, 1::2] << 4))


@pytest.mark.gpu
def test_packers_bit_exact(cuda):
    from mzoo_b200 import kvcache
    g = torch.Generator().manual_seed(3)
    inputs = [_bf16(x) for x, *_ in _cases()]
    inputs.append((torch.randn(2, 300, 1, 128, generator=g) * 3).to(torch.bfloat16))
    for xb in inputs:
        c8, s8, d8 = K.pack_window(xb)
        gc8, gs8 = kvcache.pack_window(xb.to(cuda))
        assert torch.equal(gc8.cpu(), c8) and torch.equal(gs8.cpu(), s8)
        assert torch.equal(kvcache.unpack_window(gc8, gs8).cpu().view(torch.int16), d8.view(torch.int16))
        c4, s4, d4 = K.pack_main(xb)
        gc4, gs4 = kvcache.pack_main(xb.to(cuda))
        assert torch.equal(gc4.cpu(), c4) and torch.equal(gs4.cpu(), s4)
        assert torch.equal(kvcache.unpack_main(gc4, gs4).cpu().view(torch.int16), d4.view(torch.int16))


@pytest.mark.gpu
def test_csa2_fp_attn_equals_csa2_on_dequantised(cuda):
    """Same inputs, same numbers: forward, backward and the autograd wrapper."""
    from mzoo_b200 import csa2_attn, csa2_fp_attn, kvcache
    g = torch.Generator().manual_seed(5)
    B, S, H, D, G, topk, ratio = 2, 192, 16, 128, 48, 24, 4
    q = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(cuda)
    kv = torch.randn(B, S, 1, D, generator=g).to(torch.bfloat16).to(cuda)
    main = torch.randn(B, G, 1, D, generator=g).to(torch.bfloat16).to(cuda)
    idx = torch.full((B, S, topk), -1, dtype=torch.int32)
    for b in range(B):
        for s in range(S):
            vis = min(G, (s + 1) // ratio)
            sel = torch.sort(torch.randperm(vis, generator=g)[:topk]).values
            idx[b, s, :len(sel)] = sel
    idx = idx.to(cuda)
    sinks = torch.randn(H, generator=g).to(cuda)
    kc, ks = kvcache.pack_window(kv)
    mc, ms = kvcache.pack_main(main)
    kv_d, main_d = kvcache.unpack_window(kc, ks), kvcache.unpack_main(mc, ms)
    o, lse = csa2_fp_attn.fwd(q, kc, ks, mc, ms, idx, window=64, compress_ratio=ratio, sinks=sinks)
    o_ref, lse_ref = csa2_attn.fwd(q, kv_d, main_d, idx, window=64, compress_ratio=ratio, sinks=sinks)
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)
    do = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(cuda)
    got = csa2_fp_attn.bwd(q, kc, ks, mc, ms, idx, o, lse, do, window=64, compress_ratio=ratio, sinks=sinks)
    ref = csa2_attn.bwd(q, kv_d, main_d, idx, o_ref, lse_ref, do, window=64, compress_ratio=ratio, sinks=sinks)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    assert (got[2].float() - ref[2].float()).abs().max() <= 2e-2  # dmain: fp32 atomics, order varies
    assert torch.allclose(got[3], ref[3])
    # the QAT wrapper: latents in, gradients straight through the quantisers
    leaves = [t.detach().clone().requires_grad_() for t in (q, kv, main)]
    out = csa2_fp_attn.attn(*leaves, idx, window=64, compress_ratio=ratio, sinks=sinks)
    assert torch.equal(out.detach(), o)
    out.backward(do)
    assert torch.equal(leaves[0].grad, ref[0]) and torch.equal(leaves[1].grad, ref[1])
