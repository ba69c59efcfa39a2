"""Test configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (B200) and the built
`libaicas_decode.so`; everything else runs on the CPU.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "aicasgc-2026_b200"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built sm_100a library")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda", 0)
