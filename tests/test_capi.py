"""The C-ABI library loads on a host without a GPU and exports exactly the entry points
``include/mzb200.h`` declares (no compute calls here)."""

import ctypes
import os
import re
import subprocess

from conftest import ROOT


def _declared() -> set:
    src = open(os.path.join(ROOT, "include", "mzb200.h")).read()
    return set(re.findall(r"MZB_API\s+[\w\s\*]+?\b(mzb_\w+)\s*\(", src))


def test_header_declares_symbols():
    names = _declared()
    assert {"mzb_last_error", "mzb_version", "mzb_fq_fp4", "mzb_fq_fp8"} <= names


def test_library_exports_every_declared_symbol():
    from mzoo_b200 import build, _lib
    path = build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mzb_\w+)", out))
    assert _declared() == exported, (f"header-only: {sorted(_declared() - exported)}, "
                                     f"library-only: {sorted(exported - _declared())}")
    # the ctypes binding covers the same set and loads without a driver
    assert set(_lib.SIGNATURES) == _declared()
    lib = _lib.lib()
    assert lib.mzb_version() == 1
    assert isinstance(lib.mzb_last_error(), bytes)


def test_header_compiles_as_c():
    hdr = os.path.join(ROOT, "include", "mzb200.h")
    r = subprocess.run(["gcc", "-x", "c", "-fsyntax-only", "-Wall", "-Werror", hdr], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_shape_errors_need_no_gpu():
    """Host-side validation runs before any launch: a non-divisible block is rejected
    with MZB_ERR_SHAPE and a message, without touching the device."""
    from mzoo_b200 import _lib
    lib = _lib.lib()
    st = lib.mzb_fq_fp8(None, None, 2, 40, 0, 32, 0, None)
    assert st == _lib.MZB_ERR_SHAPE
    assert b"divisible" in lib.mzb_last_error()
    assert lib.mzb_fq_fp4(None, None, 1, 32, 0, 32, 7, None) == _lib.MZB_ERR_UNSUPPORTED
