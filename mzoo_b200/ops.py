"""``torch.library`` custom ops ``mzb::*`` -- the only place Python calls the C ABI.

Each op checks device / dtype / contiguity on the host, allocates its outputs with
torch (the library never allocates), passes raw pointers and the current stream to
``libmzb200.so`` and raises on a non-zero status.  Every op has a fake (meta)
implementation so it traces under ``torch.compile`` / ``FakeTensor`` without running.
"""

import torch

from . import _lib
from ._lib import call, ptr, require_cuda, stream_ptr


def _rows_n(x: torch.Tensor) -> tuple:
    n = x.shape[-1] if x.dim() else 1
    return (x.numel() // n if n else 0), n


# ----------------------------------------------------------------------------- fake quant

@torch.library.custom_op("mzb::fq_fp4", mutates_args=())
def fq_fp4(x: torch.Tensor, block_size: int, rule: int) -> torch.Tensor:
    require_cuda(x)
    assert x.dtype in _lib.DTYPE_CODE, f"fake quant supports fp32/bf16/fp16, got {x.dtype}"
    x = x.contiguous()
    y = torch.empty_like(x)
    rows, n = _rows_n(x)
    call("mzb_fq_fp4", ptr(x), ptr(y), rows, n, _lib.DTYPE_CODE[x.dtype], block_size, rule, stream_ptr(x.device))
    return y


@fq_fp4.register_fake
def _(x, block_size, rule):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("mzb::fq_fp8", mutates_args=())
def fq_fp8(x: torch.Tensor, block_size: int, rule: int) -> torch.Tensor:
    require_cuda(x)
    assert x.dtype in _lib.DTYPE_CODE, f"fake quant supports fp32/bf16/fp16, got {x.dtype}"
    x = x.contiguous()
    y = torch.empty_like(x)
    rows, n = _rows_n(x)
    call("mzb_fq_fp8", ptr(x), ptr(y), rows, n, _lib.DTYPE_CODE[x.dtype], block_size, rule, stream_ptr(x.device))
    return y


@fq_fp8.register_fake
def _(x, block_size, rule):
    return torch.empty_like(x, memory_format=torch.contiguous_format)
