"""pytest configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on a host without a GPU (oracle vs golden fixtures, host logic,
C-ABI symbol checks, gloo multi-rank tests); ``-m gpu`` runs the CUDA parity tests.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mzoo_b200 import build
    build.build()
    return torch.device("cuda", 0)
