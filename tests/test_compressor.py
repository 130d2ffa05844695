"""Compressor producer step: the oracle pinned to the reference's own module and functions
(CPU), the fused sm_100a kernel against the oracle and the golden vectors (GPU).

Tolerance: the bf16 latent within two bf16 units (rtol 2^-6) plus 1e-5 absolute of the
oracle, on the RMS-normalised scale, with fewer than 1 % of the values off the oracle's
bits.  The pool's softmax-weighted sum is fp32 here and float64 in the oracle: a pooled value
on a rounding boundary can take the other bf16 neighbour at the first cast, and the RMSNorm
and the bf16 weight multiply carry that unit through two more bf16 roundings (two units at
the output); where the pool's terms cancel, the last fp32 bits of a near-zero sum move by
more than a unit of that small value, which the absolute term covers; the cache entry (rope + MXFP4 fake quant) is
bit-exact against the oracle applied to the kernel's own latent, and bit-exact against the
reference wherever the latents agree.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import compressor as Cm
from oracle import quant as Q


def _cases():
    d = np.load(os.path.join(GOLDEN, "compressor.npz"))
    n = len([k for k in d.files if k.endswith(".params")])
    for c in range(n):
        key = f"c{c}."
        yield {k[len(key):]: d[k] for k in d.files if k.startswith(key)}


def _check_latent(lat_bits: np.ndarray, ref_bits: np.ndarray) -> None:
    a, b = Q.bf16_to_f32(lat_bits), Q.bf16_to_f32(ref_bits)
    np.testing.assert_allclose(a, b, rtol=2.0**-6, atol=1e-5)
    assert (lat_bits != ref_bits).mean() < 0.01


# ----------------------------------------------------------------------------- CPU: oracle pin

def test_oracle_matches_reference_golden():
    for case in _cases():
        ratio, _ = (int(x) for x in case["params"])
        lat = Cm.latent_ref(case["kv"], case.get("gate"), case["norm_w"], 1e-6, ratio)
        assert np.array_equal(lat, case["latent"])
        assert np.array_equal(Cm.rope_ref(case["latent"], case["cos"], case["sin"]), case["rotated"])
        assert np.array_equal(Cm.cache_ref(case["latent"], case["cos"], case["sin"]), case["cache"])


# ----------------------------------------------------------------------------- GPU

def _run(cuda, kv, gate, w_bits, ratio, cos, sin):
    import torch
    from mzoo_b200 import compressor as K
    t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(cuda)  # noqa: E731
    w = torch.from_numpy(w_bits.view(np.int16)).view(torch.bfloat16).to(cuda)
    lat, cache = K.compress(t(kv), t(gate), w, ratio, 1e-6, t(cos), t(sin))
    bits = lambda x: x.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    return bits(lat), (bits(cache) if cache is not None else None)


@pytest.mark.gpu
def test_kernel_matches_reference_golden(cuda):
    for case in _cases():
        ratio, _ = (int(x) for x in case["params"])
        lat, cache = _run(cuda, case["kv"], case.get("gate"), case["norm_w"], ratio, case["cos"], case["sin"])
        _check_latent(lat, case["latent"])
        assert np.array_equal(cache, Cm.cache_ref(lat, case["cos"], case["sin"]))
        same = (lat == case["latent"]).all(axis=-1)
        assert np.array_equal(cache[same], case["cache"][same])


@pytest.mark.gpu
@pytest.mark.parametrize("B,G,ratio,D,rope", [
    (2, 300, 4, 576, 64),    # the V4.1 latent: 512 nope + 64 rope, ratio 4
    (1, 64, 128, 512, 64),   # a long pool
    (3, 50, 1, 128, 32),     # ratio 1: no gate
    (1, 17, 2, 16, 4),       # smallest head_dim
    (1, 8, 4, 4096, 64),     # 1024 threads per group
])
def test_kernel_matches_oracle(cuda, B, G, ratio, D, rope):
    rng = np.random.default_rng(B * 1000 + G + D)
    kv = rng.standard_normal((B, G * ratio, D)).astype(np.float32)
    gate = (rng.standard_normal((B, G * ratio, D)) * 2).astype(np.float32) if ratio > 1 else None
    w = Q.f32_to_bf16((1 + 0.25 * rng.standard_normal(D)).astype(np.float32))
    ang = rng.uniform(0, 6, (B, G, rope // 2))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    lat, cache = _run(cuda, kv, gate, w, ratio, cos, sin)
    ref = Cm.latent_ref(kv, gate, w, 1e-6, ratio)
    _check_latent(lat, ref)
    assert np.array_equal(cache, Cm.cache_ref(lat, cos, sin))


@pytest.mark.gpu
def test_latent_only_and_shape_errors(cuda):
    import torch
    from mzoo_b200 import compressor as K
    kv = torch.randn(1, 8, 64, device=cuda)
    gate = torch.randn(1, 8, 64, device=cuda)
    w = torch.ones(64, dtype=torch.bfloat16, device=cuda)
    lat, cache = K.compress(kv, gate, w, 4)
    assert lat.shape == (1, 2, 64) and cache is None
    with pytest.raises(AssertionError, match="multiple of 16"):
        K.compress(torch.randn(1, 4, 40, device=cuda), torch.randn(1, 4, 40, device=cuda),
                   torch.ones(40, dtype=torch.bfloat16, device=cuda), 4)
    with pytest.raises(AssertionError, match="needs the gate"):
        K.compress(kv, None, w, 4)
