"""CPU restatement of the KV-cache formats -- test infrastructure, not the product.

The model's cache quantisers (``archs/dsv4/modeling_deepseek_v41.py:359-402`` for
``_pow2_ceil_scale`` / ``_e2m1_codes`` / ``_fake_quant_fp4_block``, ``:668-683`` for
``_fake_quant_fp8_block``) written to return the stored codes and scale bytes as well as
the dequantised values, in torch on the CPU.  Pinned to fixtures produced by the model's
own functions (``tests/golden/kvcache.npz``, ``make_golden.py::make_kvcache``).
"""

import torch

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def pack_window(x: torch.Tensor) -> tuple:
    """bf16/fp32 [..., D] -> (e4m3 codes uint8 [..., D], ue8m0 bytes uint8 [..., D/32],
    dequantised bf16 [..., D]) -- ``_fake_quant_fp8_block(x, 32)``."""
    D = x.shape[-1]
    b = x.float().reshape(*x.shape[:-1], D // 32, 32)
    amax = b.abs().amax(-1).clamp_min(1e-4)
    t = (amax * (1.0 / 448.0)).contiguous()
    bits = t.view(torch.int32)
    ebyte = ((bits >> 23) & 0xFF) + ((bits & 0x7FFFFF) != 0).to(torch.int32)   # k + 127
    scale = torch.exp2((ebyte - 127).to(torch.float32))
    q = (b / scale.unsqueeze(-1)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    deq = (q.float() * scale.unsqueeze(-1)).reshape(x.shape).to(torch.bfloat16)
    return q.view(torch.uint8).reshape(x.shape), ebyte.to(torch.uint8), deq


def pack_main(x: torch.Tensor) -> tuple:
    """bf16/fp32 [..., D] -> (packed e2m1 uint8 [..., D/2] (low nibble first), e4m3 bytes
    uint8 [..., D/16], dequantised bf16 [..., D]) -- ``_fake_quant_fp4_block(x, 16, True)``."""
    D = x.shape[-1]
    b = x.float().reshape(*x.shape[:-1], D // 16, 16)
    amax = b.abs().amax(-1)
    scale = (amax.clamp_min(6.0 * 2.0**-9) / 6.0).to(torch.float8_e4m3fn)
    q = (b / scale.float().unsqueeze(-1)).clamp(-6.0, 6.0)
    mag, neg = q.abs(), torch.signbit(q)
    thr = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    ties_up = torch.tensor([False, True, False, True, False, True, False])
    thr = torch.where(ties_up, thr, torch.nextafter(thr, torch.full_like(thr, float("inf"))))
    code = (mag.unsqueeze(-1) >= thr).sum(-1).to(torch.uint8) | (neg.to(torch.uint8) << 3)
    vals = _E2M1[(code & 7).long()] * torch.where((code & 8).bool() & (code & 7 != 0), -1.0, 1.0)
    deq = (vals * scale.float().unsqueeze(-1)).reshape(x.shape).to(torch.bfloat16)
    code = code.reshape(*x.shape[:-1], D)
    packed = code[..., 0::2] | (code[..., 1::2] << 4)
    return packed, scale.view(torch.uint8), deq
