"""Test configuration.

Markers:
  gpu   — needs a B200 (sm_100a); run with ``-m gpu`` on the GPU box.
  slow  — long CPU oracle runs.
CPU tests (``-m "not gpu"``) cover the oracle against the reference's pinned
properties and the committed golden fixtures, the host logic, and that the
C-ABI library loads and exports every declared symbol.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "slow: long-running oracle case")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def built_lib():
    """Build libtitan_moe.so if needed (nvcc cross-compiles without a GPU)."""
    from titan_b200 import build
    build.build()
    from titan_b200 import _lib
    return _lib


@pytest.fixture(scope="session")
def cuda(built_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
