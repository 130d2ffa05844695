"""Fused RMSNorm + RoPE prologue of q / kv (``layers/attn/norm_rope.py``): the oracle pinned
to the model's own ``DeepseekV41RMSNorm`` + ``apply_rotary_pos_emb`` (CPU), and the
sm_100a kernels against it under the reference's criterion (``norm_rope_test.py:45-69``):
the kernel's error to the fp32 composition is at most 2x that of the same composition
run in bf16, for the output and both gradients."""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import norm_rope as N
from oracle.quant import bf16_to_f32

CASES = 4


def _golden():
    return np.load(os.path.join(GOLDEN, "norm_rope.npz"))


def _f(d, key):
    v = d[key]
    return bf16_to_f32(v) if v.dtype == np.uint16 else v.astype(np.float32)


@pytest.mark.parametrize("c", range(CASES))
def test_oracle_matches_model_fp32(c):
    d, k = _golden(), f"c{c}."
    out, _ = N.norm_rope_fwd(_f(d, k + "f32.x"), _f(d, k + "f32.w"), d[k + "cos"], d[k + "sin"])
    np.testing.assert_allclose(out, d[k + "f32.y"], rtol=0, atol=2e-5)
    dx, dw = N.norm_rope_bwd(_f(d, k + "f32.x"), _f(d, k + "f32.w"), d[k + "cos"], d[k + "sin"], d[k + "dy"])
    np.testing.assert_allclose(dx, d[k + "dx"], rtol=0, atol=1e-4)
    np.testing.assert_allclose(dw, d[k + "dw"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("c", range(CASES))
def test_oracle_matches_model_bf16(c):
    """Same rounding points as the model's bf16 composition: equal up to one bf16 step
    where the fp32 mean's summation order moves rstd across a rounding boundary."""
    d, k = _golden(), f"c{c}."
    out, _ = N.norm_rope_fwd(_f(d, k + "bf16.x"), _f(d, k + "bf16.w"), d[k + "cos"], d[k + "sin"], dtype="bf16")
    ref = _f(d, k + "bf16.y")
    step = np.abs(ref) * 2.0**-7 + 1e-30
    assert (np.abs(out - ref) <= step).all()
    assert (out == ref).mean() > 0.99


def _within_2x(got, ref, base, what):
    e_got = np.abs(got - ref).max()
    e_base = np.abs(base - ref).max()
    print(f"{what}: kernel err {e_got:.3e}, torch-bf16 err {e_base:.3e}")
    assert e_got <= 2 * e_base + 1e-6, what


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(2, 512, 4, 64, 16), (2, 512, 1, 64, 16), (1, 256, 1, 128, 64),
                                   (1, 256, 64, 128, 64), (3, 331, 5, 96, 24), (1, 64, 8, 256, 64)], ids=str)
def test_kernel_fwd_bwd_within_2x_bf16(cuda, shape):
    import torch
    from mzoo_b200 import norm_rope
    B, S, H, D, rd = shape
    g = torch.Generator(device="cpu").manual_seed(B * S + D)
    x = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S, dtype=torch.float32)
    freqs = pos[:, None] / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    cos, sin = freqs.cos()[None].expand(B, -1, -1), freqs.sin()[None].expand(B, -1, -1)
    dy = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    xg, wg = x.to(cuda).requires_grad_(), w.to(cuda).requires_grad_()
    out = norm_rope.qk_norm_rope(xg, wg, cos.to(cuda), sin.to(cuda))
    out.backward(dy.to(cuda))
    xf, wf, dyf = x.float().numpy(), w.float().numpy(), dy.float().numpy()
    cn, sn = cos.numpy(), sin.numpy()
    ref, _ = N.norm_rope_fwd(xf, wf, cn, sn)                      # fp32 composition
    base, _ = N.norm_rope_fwd(xf, wf, cn, sn, dtype="bf16")       # the same in bf16
    _within_2x(out.detach().float().cpu().numpy(), ref, base, "out")
    rdx, rdw = N.norm_rope_bwd(xf, wf, cn, sn, dyf)
    # gradients: bf16 outputs of an fp32 computation -- within one bf16 step of the exact
    # closed form (plus fp32 noise); dw (fp32 sum over rows, returned in the weight dtype) too
    gdx = xg.grad.float().cpu().numpy()
    assert (np.abs(gdx - rdx) <= 2.0**-7 * np.abs(rdx) + 1e-4 * np.abs(rdx).max()).all(), "dx"
    gdw = wg.grad.float().cpu().numpy()
    assert (np.abs(gdw - rdw) <= 2.0**-7 * np.abs(rdw) + 1e-4 * np.abs(rdw).max()).all(), "dw"


@pytest.mark.gpu
def test_kernel_rstd_and_determinism(cuda):
    """The forward's saved rstd equals the oracle's; the backward's dw (two-stage
    fixed-order reduction, no atomics) is bitwise reproducible."""
    import torch
    from mzoo_b200 import norm_rope
    B, S, H, D, rd = 2, 300, 16, 128, 64
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(cuda)
    w = torch.randn(D, generator=g).to(torch.bfloat16).to(cuda)
    cos = torch.rand(B, S, rd // 2, generator=g).to(cuda)
    sin = torch.rand(B, S, rd // 2, generator=g).to(cuda)
    out, rstd = norm_rope.fwd(x, w, cos, sin)
    _, ref_rstd = N.norm_rope_fwd(x.float().cpu().numpy(), w.float().cpu().numpy(), cos.cpu().numpy(),
                                  sin.cpu().numpy())
    np.testing.assert_allclose(rstd.cpu().numpy().reshape(ref_rstd.shape), ref_rstd, rtol=1e-6)
    dy = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(cuda)
    a = norm_rope.bwd(x, w, cos, sin, rstd, dy)
    b = norm_rope.bwd(x, w, cos, sin, rstd, dy)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
