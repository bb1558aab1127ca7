"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked gpu need a CUDA device and call the library through its C ABI; everything else runs
on the CPU (oracle against golden fixtures and the compiled reference, ABI exports, host logic).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")
    config.addinivalue_line("markers", "slow: full-size configs (minutes)")


@pytest.fixture(scope="session")
def executor():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import xspmm_b200 as xs
    return xs.CudaExecutor(0)
