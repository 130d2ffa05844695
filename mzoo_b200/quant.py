"""Fake-quant (quantise -> dequantise) with mzoo's call signatures, on sm_100a kernels.

Drop-in for ``src/mzoo/archs/owlet1/quant.py`` (``_fake_quant_fp4_block`` :49,
``_fake_quant_fp8_block`` :72; same functions in
``archs/dsv4/modeling_deepseek_v41.py:383,616``): same arguments, same output dtype,
bit-identical values, and -- like the reference -- a last dimension that the block size
does not divide returns ``x`` itself unchanged.

Extra rules (not in mzoo):
- ``fake_quant_fp4_block(x, 32, rule="ocp")`` -- OCP MXFP4: e8m0 scale
  ``2^(floor(log2 amax) - 2)``, e2m1 round-to-nearest-even, saturating at +-6.
- ``fake_quant_fp8_block(x, 128, rule="absmax")`` -- e4m3 with scale ``amax / 448`` per tile.

``*_ste`` variants return the quantised values with an identity gradient (the
straight-through estimator of ``indexer/attn.py:29-34``), in one kernel launch.
"""

import torch

from . import ops

_FP4_RULES = {"mzoo": None, "ocp": 2}
_FP8_RULES = {"mzoo": 0, "absmax": 1}


def _fp4_rule(e4m3_scales: bool, rule: str) -> int:
    assert rule in _FP4_RULES, f"unknown fp4 rule {rule!r} (have {sorted(_FP4_RULES)})"
    if rule == "ocp":
        assert not e4m3_scales, "the OCP rule has e8m0 scales only"
        return 2
    return 1 if e4m3_scales else 0


def fake_quant_fp4_block(x: torch.Tensor, block_size: int = 32, *, e4m3_scales: bool = False,
                         rule: str = "mzoo") -> torch.Tensor:
    """Block-wise fp4 (e2m1) fake quantisation along the last dim."""
    code = _fp4_rule(e4m3_scales, rule)
    if x.shape[-1] % block_size:
        return x  # quant.py:55-56: shapes the reference cannot block run unquantised
    return ops.fq_fp4(x, block_size, code)


def fake_quant_fp8_block(x: torch.Tensor, block_size: int = 32, *, rule: str = "mzoo") -> torch.Tensor:
    """Block-wise fp8 (e4m3) fake quantisation along the last dim."""
    assert rule in _FP8_RULES, f"unknown fp8 rule {rule!r} (have {sorted(_FP8_RULES)})"
    if x.shape[-1] % block_size:
        return x  # quant.py:79-80
    return ops.fq_fp8(x, block_size, _FP8_RULES[rule])


def _fake_quant_fp4_block(x: torch.Tensor, block_size: int, e4m3_scales: bool = False) -> torch.Tensor:
    """Reference signature (quant.py:49)."""
    return fake_quant_fp4_block(x, block_size, e4m3_scales=e4m3_scales)


def _fake_quant_fp8_block(x: torch.Tensor, block_size: int = 32) -> torch.Tensor:
    """Reference signature (quant.py:72)."""
    return fake_quant_fp8_block(x, block_size)


class _Ste(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fn):
        return fn(x.detach())

    @staticmethod
    def backward(ctx, g):
        return g, None


def fake_quant_fp4_ste(x: torch.Tensor, block_size: int = 32, *, e4m3_scales: bool = False,
                       rule: str = "mzoo") -> torch.Tensor:
    """fp4 round trip with a straight-through gradient (``indexer/attn.py:29``)."""
    return _Ste.apply(x, lambda t: fake_quant_fp4_block(t, block_size, e4m3_scales=e4m3_scales, rule=rule))


def fake_quant_fp8_ste(x: torch.Tensor, block_size: int = 32, *, rule: str = "mzoo") -> torch.Tensor:
    """fp8 round trip with a straight-through gradient."""
    return _Ste.apply(x, lambda t: fake_quant_fp8_block(t, block_size, rule=rule))
