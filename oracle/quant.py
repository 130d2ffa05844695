"""Fake-quant oracle (numpy) -- test infrastructure, not the product.

Restates ``src/mzoo/archs/owlet1/quant.py`` (identical to
``src/mzoo/archs/dsv4/modeling_deepseek_v41.py:343-402,613-630``) in float32 numpy with
the same rounding at every step, plus the two rules BASELINE config 5 names that the
reference does not implement (OCP MXFP4 and FP8 per-tile absmax).

Every function takes and returns numpy arrays; ``dtype`` of the output equals the
input's (float32, or a bfloat16 stand-in given as ``uint16`` bit patterns -- see
``bf16_to_f32`` / ``f32_to_bf16``).
"""

import numpy as np

FP4_MAX = np.float32(6.0)
FP8_MAX = np.float32(448.0)
# e2m1 code -> value, sign in bit 3 (quant.py:8-11). Code 8 (negative zero) is +0.0.
FP4_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


# ----------------------------------------------------------------------------- bf16 helpers

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bfloat16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bfloat16 bits, round-to-nearest-even; NaN stays NaN (quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return out


# ----------------------------------------------------------------------------- scalar rules

def pow2_ceil_scale(t: np.ndarray) -> np.ndarray:
    """``2^ceil(log2 t)`` for float32 ``t > 0`` through the exponent bits, exactly like
    ``_pow2_ceil_scale`` (quant.py:23-31): exponent - 127 + (mantissa != 0)."""
    bits = np.ascontiguousarray(t, dtype=np.float32).view(np.int32)
    exponent = (bits >> 23) & 0xFF
    mantissa = bits & 0x7FFFFF
    k = exponent - 127 + (mantissa != 0).astype(np.int32)
    return np.exp2(k.astype(np.float64)).astype(np.float32)


def e4m3_round(v: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn -> float32, the value torch's ``.to(torch.float8_e4m3fn)``
    produces (``torch/headeronly/util/Float8_e4m3fn.h`` ``fp8e4m3fn_from_fp32_value``):
    round-to-nearest-even; |v| >= 480 and NaN give NaN, and (464, 480) rounds onto the
    NaN code as well; [448, 464] gives 448; below 2^-6 the grid is 2^-9 (subnormals)."""
    v = np.asarray(v, dtype=np.float32).astype(np.float64)
    a = np.abs(v)
    out = np.empty_like(a)
    sub = a < 2.0**-6
    out[sub] = np.rint(a[sub] / 2.0**-9) * 2.0**-9
    nrm = ~sub & np.isfinite(a)
    e = np.floor(np.log2(np.where(nrm, a, 1.0)))
    # guard log2 rounding at exact powers of two
    e = np.where(np.exp2(e) > a, e - 1, e)
    e = np.where(np.exp2(e + 1) <= a, e + 1, e)
    step = np.exp2(e - 3)
    out[nrm] = (np.rint(a / step) * step)[nrm]
    out[(out > 448.0) | ~np.isfinite(a)] = np.nan
    return np.copysign(out, v).astype(np.float32)


def e2m1_codes(q: np.ndarray) -> np.ndarray:
    """``_e2m1_codes`` (quant.py:34-46): count of thresholds passed, sign in bit 3.
    Ties at 0.25 / 1.25 / 2.5 / 5.0 round down, at 0.75 / 1.75 / 3.5 round up."""
    q = np.asarray(q, dtype=np.float32)
    mag = np.abs(q)
    neg = np.signbit(q)
    bnd = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    ties_up = np.array([False, True, False, True, False, True, False])
    thr = np.where(ties_up, bnd, np.nextafter(bnd, np.float32(np.inf)))
    codes = (mag[..., None] >= thr).sum(-1).astype(np.uint8)
    return codes | (neg.astype(np.uint8) << 3)


def _clamp(v: np.ndarray, lo: float, hi: float) -> np.ndarray:
    """torch.clamp: NaN passes through."""
    return np.where(v < lo, np.float32(lo), np.where(v > hi, np.float32(hi), v)).astype(np.float32)


# ----------------------------------------------------------------------------- block quantisers

def _as_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    return bf16_to_f32(x) if dtype == "bf16" else np.asarray(x, dtype=np.float32)


def _from_f32(y: np.ndarray, dtype: str) -> np.ndarray:
    return f32_to_bf16(y) if dtype == "bf16" else y.astype(np.float32)


def fake_quant_fp4(x: np.ndarray, block_size: int, rule: str = "ue8m0", dtype: str = "f32") -> np.ndarray:
    """fp4 (e2m1) quant-dequant along the last axis in blocks of ``block_size``.

    rule ``"ue8m0"``  : ``_fake_quant_fp4_block(x, bs)`` (quant.py:49-66): scale
                        ``2^ceil(log2(max(amax, 6*2^-126) * (1/6)))``.
    rule ``"e4m3"``   : ``_fake_quant_fp4_block(x, bs, e4m3_scales=True)``: scale
                        ``e4m3(max(amax, 6*2^-9) / 6)``.
    rule ``"ocp"``    : OCP MX rule: scale
                        ``2^(floor(log2 amax) - 2)`` (e8m0, exponent clamped to [-127, 127];
                        amax == 0 gives scale 1), elements saturate at +-6.
    A last axis not divisible by ``block_size`` is returned unchanged (quant.py:55-56).
    """
    n = x.shape[-1]
    if n % block_size:
        return x
    xf = _as_f32(x, dtype)
    blocks = xf.reshape(*xf.shape[:-1], n // block_size, block_size)
    amax = np.abs(blocks).max(-1).astype(np.float32)
    if rule == "e4m3":
        scale = e4m3_round(np.maximum(amax, np.float32(6.0 * 2.0**-9)) / FP4_MAX)
    elif rule == "ue8m0":
        scale = pow2_ceil_scale(np.maximum(amax, np.float32(6.0 * 2.0**-126)) * np.float32(1.0 / 6.0))
    elif rule == "ocp":
        bits = amax.view(np.int32)
        exp = ((bits >> 23) & 0xFF).astype(np.int64)
        # floor(log2 amax): normal -> exponent-127; subnormal -> position of the top set bit
        man = (bits & 0x7FFFFF).astype(np.int64)
        sub_fl = np.where(man > 0, np.floor(np.log2(np.maximum(man, 1))).astype(np.int64) - 149, -127)
        fl = np.where(exp > 0, exp - 127, sub_fl)
        e = np.clip(fl - 2, -127, 127)
        scale = np.where(amax > 0, np.exp2(e.astype(np.float64)), 1.0).astype(np.float32)
    else:
        raise ValueError(rule)
    q = _clamp((blocks / scale[..., None]).astype(np.float32), -6.0, 6.0)
    vals = FP4_TABLE[e2m1_codes(q).astype(np.int64)]
    y = (vals * scale[..., None]).astype(np.float32).reshape(xf.shape)
    return _from_f32(y, dtype)


def fake_quant_fp8(x: np.ndarray, block_size: int = 32, rule: str = "ue8m0", dtype: str = "f32") -> np.ndarray:
    """fp8 (e4m3) quant-dequant along the last axis in blocks of ``block_size``.

    rule ``"ue8m0"``  : ``_fake_quant_fp8_block(x, bs)`` (quant.py:72-86): amax clamped to
                        1e-4, scale ``2^ceil(log2(amax * (1/448)))``, values clamped to
                        +-448 then cast to e4m3 (RTNE).
    rule ``"absmax"`` : per-tile absmax (tile = ``block_size``):
                        scale ``amax / 448`` (1 when amax == 0), values clamped to +-448.
    """
    n = x.shape[-1]
    if n % block_size:
        return x
    xf = _as_f32(x, dtype)
    blocks = xf.reshape(*xf.shape[:-1], n // block_size, block_size)
    amax = np.abs(blocks).max(-1).astype(np.float32)
    if rule == "ue8m0":
        scale = pow2_ceil_scale(np.maximum(amax, np.float32(1e-4)) * np.float32(1.0 / 448.0))
    elif rule == "absmax":
        scale = (amax / FP8_MAX).astype(np.float32)
        scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    else:
        raise ValueError(rule)
    q = _clamp((blocks / scale[..., None]).astype(np.float32), -448.0, 448.0)
    y = (e4m3_round(q) * scale[..., None]).astype(np.float32).reshape(xf.shape)
    return _from_f32(y, dtype)


def quantize_fp8_rows(x: np.ndarray, tile: int) -> tuple:
    """Absmax FP8 quantisation used by the synthetic inputs of the indexer / latent
    configs: per ``tile`` elements of the last axis, ``scale = amax / 448`` (1 if 0),
    codes = e4m3(x / scale).  Returns (codes as float32 values on the e4m3 grid,
    float32 scales [..., n/tile])."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    blocks = x.reshape(*x.shape[:-1], n // tile, tile)
    amax = np.abs(blocks).max(-1).astype(np.float32)
    scale = np.where(amax > 0, amax / FP8_MAX, np.float32(1.0)).astype(np.float32)
    q = _clamp((blocks / scale[..., None]).astype(np.float32), -448.0, 448.0)
    return e4m3_round(q).reshape(x.shape), scale
