"""Failure detection without a GPU fault: every device wait in the kernels is bounded and
reports a site code through the error word instead of hanging.  Here a wait that nothing
satisfies (``mzb_selftest_bounded_wait``) runs out after a short limit; the kernel returns,
the code reaches the host through both the checked and the deferred (``check_errors``)
paths, and the context keeps working afterwards."""

import pytest


@pytest.mark.gpu
@pytest.mark.parametrize("scope,code", [(0, 901), (1, 902)])
def test_wait_runs_out_and_reports(cuda, scope, code):
    import torch
    from mzoo_b200 import ops
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    got = ops.selftest_bounded_wait(cuda, 2_000_000, scope, check=True)  # 2 ms limit
    e.record()
    torch.cuda.synchronize()
    assert got == code
    assert 1.5 <= s.elapsed_time(e) < 1000.0, "the wait neither ran out on time nor returned"


@pytest.mark.gpu
def test_deferred_error_word_and_context_still_usable(cuda):
    import torch
    import mzoo_b200
    from mzoo_b200 import _lib, ops, quant
    mzoo_b200.check_errors()  # start clean
    assert ops.selftest_bounded_wait(cuda, 1_000_000, 0, check=False) == 0  # no host sync
    with pytest.raises(_lib.MzbError, match="901"):
        mzoo_b200.check_errors()
    mzoo_b200.check_errors()  # the word was cleared
    x = torch.randn(64, 128, device=cuda)
    y = quant._fake_quant_fp8_block(x, 32)
    assert torch.isfinite(y).all() and (y - x).abs().max() < 0.1 * x.abs().max()


def test_selftest_rejects_bad_limits():
    from mzoo_b200 import _lib
    import ctypes
    lib = _lib.lib()
    assert lib.mzb_selftest_bounded_wait(0, 0, ctypes.c_void_p(16), None) == _lib.MZB_ERR_SHAPE
    assert lib.mzb_selftest_bounded_wait(3_000_000_000, 0, ctypes.c_void_p(16), None) == _lib.MZB_ERR_SHAPE
    assert lib.mzb_selftest_bounded_wait(1000, 2, ctypes.c_void_p(16), None) == _lib.MZB_ERR_SHAPE
