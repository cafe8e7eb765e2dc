"""Shared test configuration.

Markers: ``gpu`` — needs a CUDA device (a B200); everything else runs on CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


@pytest.fixture(scope="session")
def cuda_lib():
    """The product library, loaded through its C ABI (fails loudly if absent)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test ran without a CUDA device")
    from llama2_b200 import capi
    return capi.lib()
