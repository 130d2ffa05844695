"""Fake quant: oracle pinned to the reference's golden vectors (CPU), and the sm_100a
kernels bit-exact against the oracle and the golden vectors (GPU).

Reference: ``src/mzoo/archs/owlet1/quant.py:23-86``.  The reference's own tests only
check the STE forward against ``_fake_quant_fp4_block`` (``indexer/bwd_test.py:170-190``);
the hand-picked tie / clamp / subnormal cases here come from the rule as written in
``quant.py:34-46`` (ties at 0.25/1.25/2.5/5.0 down, at 0.75/1.75/3.5 up).
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import quant as Q

RULES = {  # fixture key -> (oracle fn, kernel kwargs)
    "fp4_32": (lambda x, dt: Q.fake_quant_fp4(x, 32, "ue8m0", dt), ("fp4", 32, dict())),
    "fp4_16e4m3": (lambda x, dt: Q.fake_quant_fp4(x, 16, "e4m3", dt), ("fp4", 16, dict(e4m3_scales=True))),
    "fp8_32": (lambda x, dt: Q.fake_quant_fp8(x, 32, "ue8m0", dt), ("fp8", 32, dict())),
    "fp8_16": (lambda x, dt: Q.fake_quant_fp8(x, 16, "ue8m0", dt), ("fp8", 16, dict())),
}


def _golden():
    d = np.load(os.path.join(GOLDEN, "quant.npz"))
    cases = sorted({k.rsplit(".", 1)[0] for k in d.files})
    return d, cases


def same_bits(a: np.ndarray, b: np.ndarray, dt: str) -> np.ndarray:
    """Bit equality, with any NaN equal to any NaN (payload bits differ across casts)."""
    fa = Q.bf16_to_f32(a) if dt == "bf16" else np.asarray(a, np.float32)
    fb = Q.bf16_to_f32(b) if dt == "bf16" else np.asarray(b, np.float32)
    ua = np.asarray(a).view(np.uint16 if dt == "bf16" else np.uint32)
    ub = np.asarray(b).view(ua.dtype)
    return (ua == ub) | (np.isnan(fa) & np.isnan(fb))


# ----------------------------------------------------------------------------- CPU: oracle pin

@pytest.mark.parametrize("rule", sorted(RULES))
def test_oracle_matches_reference_golden(rule):
    d, cases = _golden()
    fn = RULES[rule][0]
    for case in cases:
        dt = case.split(".")[1]
        x, ref = d[f"{case}.x"], d[f"{case}.{rule}"]
        got = fn(x, dt)
        assert same_bits(ref, got, dt).all(), f"{case} {rule}"


def test_oracle_e2m1_ties():
    q = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -5.0, 0.0, -0.0], np.float32)
    vals = Q.FP4_TABLE[Q.e2m1_codes(q).astype(np.int64)]
    np.testing.assert_array_equal(vals, [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 0.0, -1.0, -4.0, 0.0, 0.0])


def test_oracle_ocp_rule():
    """OCP MXFP4: scale 2^(floor(log2 amax) - 2); amax 6.5 -> scale 1, 7.9 saturates to 6."""
    x = np.zeros((1, 32), np.float32)
    x[0, :4] = [6.5, -7.9, 0.3, 2.6]
    y = Q.fake_quant_fp4(x, 32, "ocp")
    np.testing.assert_array_equal(y[0, :4], [6.0, -6.0, 0.5, 3.0])
    x[0, 0] = 64.0  # floor(log2 64) = 6 -> scale 16
    y = Q.fake_quant_fp4(x, 32, "ocp")
    assert y[0, 0] == 64.0 and y[0, 2] == 0.0 and y[0, 3] == 0.0


def test_oracle_fp8_absmax_rule():
    x = np.linspace(-3, 3, 128, dtype=np.float32).reshape(1, 128)
    y = Q.fake_quant_fp8(x, 128, "absmax")
    assert np.abs(y - x).max() <= 3 / 448 * 16  # one e4m3 step at the top of the range
    assert Q.fake_quant_fp8(np.zeros((1, 128), np.float32), 128, "absmax").max() == 0


def test_ragged_last_dim_passes_through():
    x = np.random.default_rng(0).standard_normal((3, 40)).astype(np.float32)
    assert Q.fake_quant_fp4(x, 32) is x and Q.fake_quant_fp8(x, 32) is x


# ----------------------------------------------------------------------------- GPU: kernels

def _kernel(rule_key, x):
    from mzoo_b200 import quant
    kind, bs, kw = RULES[rule_key][1]
    return quant.fake_quant_fp4_block(x, bs, **kw) if kind == "fp4" else quant.fake_quant_fp8_block(x, bs, **kw)


def _to_torch(a, dt, device):
    import torch
    if dt == "bf16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _to_np(t, dt):
    import torch
    t = t.detach().cpu().contiguous()
    return t.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else t.numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("rule", sorted(RULES))
def test_kernel_matches_reference_golden(cuda, rule):
    d, cases = _golden()
    for case in cases:
        dt = case.split(".")[1]
        x = d[f"{case}.x"]
        got = _to_np(_kernel(rule, _to_torch(x, dt, cuda)), dt)
        assert same_bits(d[f"{case}.{rule}"], got, dt).all(), f"{case} {rule}"


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(4, 8192, 128), (7, 96), (1, 16), (3, 5, 2048)])
def test_kernel_matches_oracle_random(cuda, dt, shape):
    rng = np.random.default_rng(sum(shape))
    x32 = (rng.standard_normal(shape) * np.exp(rng.uniform(-8, 8, shape[:-1] + (1,)))).astype(np.float32)
    x = Q.f32_to_bf16(x32) if dt == "bf16" else x32
    xt = _to_torch(x, dt, cuda)
    from mzoo_b200 import quant
    cases = [
        (quant.fake_quant_fp4_block(xt, 32), Q.fake_quant_fp4(x, 32, "ue8m0", dt)),
        (quant.fake_quant_fp4_block(xt, 16, e4m3_scales=True), Q.fake_quant_fp4(x, 16, "e4m3", dt)),
        (quant.fake_quant_fp4_block(xt, 32, rule="ocp"), Q.fake_quant_fp4(x, 32, "ocp", dt)),
        (quant.fake_quant_fp8_block(xt, 32), Q.fake_quant_fp8(x, 32, "ue8m0", dt)),
        (quant.fake_quant_fp8_block(xt, 16), Q.fake_quant_fp8(x, 16, "ue8m0", dt)),
    ]
    if shape[-1] % 128 == 0:
        cases.append((quant.fake_quant_fp8_block(xt, 128, rule="absmax"), Q.fake_quant_fp8(x, 128, "absmax", dt)))
    for i, (got, ref) in enumerate(cases):
        assert same_bits(ref, _to_np(got, dt), dt).all(), f"case {i}"


@pytest.mark.gpu
def test_kernel_odd_block_and_unaligned(cuda):
    """Block sizes that are not a power-of-two multiple of the vector width and an
    unaligned view take the scalar kernel; results are still bit-exact."""
    import torch
    from mzoo_b200 import quant
    rng = np.random.default_rng(5)
    x = rng.standard_normal((6, 48)).astype(np.float32)
    got = quant.fake_quant_fp4_block(torch.from_numpy(x).to(cuda), 24)
    assert same_bits(Q.fake_quant_fp4(x, 24), got.cpu().numpy(), "f32").all()
    big = torch.from_numpy(rng.standard_normal(1 + 64 * 4).astype(np.float32)).to(cuda)
    view = big[1:].view(4, 64)  # 4-byte offset: not 16-byte aligned
    got = quant.fake_quant_fp8_block(view, 32)
    assert same_bits(Q.fake_quant_fp8(view.cpu().numpy(), 32), got.cpu().numpy(), "f32").all()


@pytest.mark.gpu
def test_ste_forward_bits_and_identity_grad(cuda):
    """``indexer/bwd_test.py:170-190``: STE forward equals the plain quantiser bit for bit,
    gradient is the identity."""
    import torch
    from mzoo_b200 import quant
    x = torch.randn(4, 64, 128, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = quant.fake_quant_fp4_ste(x, 32)
    assert torch.equal(y, quant._fake_quant_fp4_block(x.detach(), 32))
    g = torch.randn_like(y)
    y.backward(g)
    assert torch.equal(x.grad, g)


@pytest.mark.gpu
def test_ragged_returns_input_object(cuda):
    import torch
    from mzoo_b200 import quant
    x = torch.randn(3, 40, device=cuda)
    assert quant._fake_quant_fp4_block(x, 32) is x and quant._fake_quant_fp8_block(x, 32) is x


@pytest.mark.gpu
def test_cpu_tensor_rejected(cuda):
    import torch
    from mzoo_b200 import quant
    with pytest.raises(AssertionError, match="CUDA"):
        quant._fake_quant_fp8_block(torch.randn(2, 32), 32)
