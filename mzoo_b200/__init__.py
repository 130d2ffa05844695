"""mzoo_b200: B200-native (sm_100a) kernels for mzoo's DeepSeek-V4.1 attention hot path.

Drop-in modules mirroring the reference's call signatures:

- ``mzoo_b200.quant``      fp8 / fp4 fake quant (``archs/owlet1/quant.py``)
- ``mzoo_b200.indexer``    lightning indexer fwd / bwd / top-k (``layers/attn/indexer``)
- ``mzoo_b200.swa_attn``   sliding-window latent MQA (``layers/attn/swa_attn``)
- ``mzoo_b200.csa2_attn``  window + gathered sparse latent MQA (``layers/attn/csa2_attn``)
- ``mzoo_b200.sparse_mla`` 576/512 FP8-latent sparse prefill and paged decode

All compute runs in ``libmzb200.so`` (hand-written CUDA for sm_100a) behind the C ABI
of ``include/mzb200.h``; there is no CPU fallback.

The wrappers never block the host (like the reference's): a device-side failure (a
bounded wait that gave up, a top-k error band too wide) is recorded in a per-device error
word that ``check_errors()`` reads and clears; ``check=True`` on a wrapper reads it right
after that launch instead.
"""

__version__ = "0.2.0"


def check_errors(device=None) -> None:
    """Raise ``mzoo_b200._lib.MzbError`` if a kernel recorded a device-side failure since
    the last call (synchronises with the device)."""
    from .ops import check_errors as _check
    _check(device)
