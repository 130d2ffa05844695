"""ctypes binding of ``libmzb200.so`` (the C ABI declared in ``include/mzb200.h``).

The library is built in-tree (``python -m mzoo_b200.build``).  There is no fallback:
if the shared object is missing or lacks a symbol, importing the ops fails loudly.
Tensors cross the boundary as raw device pointers (``tensor.data_ptr()``) and the
current torch CUDA stream as ``void*``.
"""

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmzb200.so")

MZB_OK = 0
MZB_ERR_SHAPE = -1
MZB_ERR_UNSUPPORTED = -2
MZB_ERR_LAUNCH = -3
MZB_ERR_TIMEOUT = -4
MZB_ERR_ALIGN = -5
MZB_ERR_BOUND = -6

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_F32 = ctypes.c_float

# name -> argtypes (every function returns int status unless listed in _RESTYPE)
SIGNATURES = {
    "mzb_last_error": [],
    "mzb_version": [],
    "mzb_fq_fp4": [_P, _P, _I64, _I64, _I32, _I32, _I32, _P],
    "mzb_fq_fp8": [_P, _P, _I64, _I64, _I32, _I32, _I32, _P],
    "mzb_indexer_scores": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I64, _F32,
                           _I32, _P, _I32, _I64, _P, _P],
    "mzb_indexer_topk": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I64,
                         _F32, _I32, _F32, _P, _I32, _I64, _P, _P],
    "mzb_indexer_bwd": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _I64, _F32, _P, _P],
    "mzb_attn_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _I32, _I64, _I32, _F32, _P, _P],
    "mzb_attn_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I64, _I64, _I32, _I32,
                     _I32, _I64, _I32, _F32, _P, _P],
    "mzb_attn_bwd_splits": [_I64, _I64, _I32, _I32],
    "mzb_sparse_mla_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I64, _I64, _I32,
                           _I32, _F32, _I32, _P, _P, _P],
    "mzb_sparse_mla_splits": [_I64],
    "mzb_sparse_mla_fwd_noalloc": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I64, _I64,
                                   _I32, _I32, _F32, _P, _P],
    "mzb_candidate_blocks": [_P, _P, _P, _P, _I64, _I64, _I32, _I32, _P],
    "mzb_candidate_topk": [_P, _P, _P, _I64, _I64, _I32, _I32, _I32, _P, _P],
    "mzb_compress": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _I32, _F32, _P],
    "mzb_selftest_bounded_wait": [_I64, _I32, _P, _P],
    "mzb_norm_rope_fwd": [_P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _F32, _P],
    "mzb_norm_rope_bwd_parts": [_I64, _I32],
    "mzb_norm_rope_bwd": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P],
    "mzb_kv_pack_fp8": [_P, _P, _P, _I64, _I32, _P],
    "mzb_kv_unpack_fp8": [_P, _P, _P, _I64, _I32, _P],
    "mzb_kv_pack_fp4": [_P, _P, _P, _I64, _I32, _P],
    "mzb_kv_unpack_fp4": [_P, _P, _P, _I64, _I32, _P],
}
_RESTYPE = {"mzb_last_error": ctypes.c_char_p}

_lib = None


class MzbError(RuntimeError):
    """A kernel-side failure reported through the C ABI (launch error, timeout, bound check)."""


def lib() -> ctypes.CDLL:
    """Load the shared library once and bind every declared symbol."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m mzoo_b200.build` "
                              "(mzoo_b200 has no CPU or eager fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError here = header/library mismatch
            fn.argtypes = argtypes
            fn.restype = _RESTYPE.get(name, ctypes.c_int)
        _lib = handle
    return _lib


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(status: int, what: str) -> None:
    """Raise on a non-zero status: shape / support / alignment errors become
    ``AssertionError`` (the reference's host-side asserts), the rest ``MzbError``."""
    if status == MZB_OK:
        return
    msg = lib().mzb_last_error().decode(errors="replace")
    if status in (MZB_ERR_SHAPE, MZB_ERR_UNSUPPORTED, MZB_ERR_ALIGN):
        raise AssertionError(f"{what}: {msg}")
    raise MzbError(f"{what} failed (status {status}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise AssertionError("mzoo_b200 kernels run on CUDA tensors only (no CPU fallback); "
                                 f"got a tensor on {t.device}")
