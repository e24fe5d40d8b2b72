"""Test configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (B200) and call the product through its
C ABI; everything else runs on the CPU (oracle pins, host logic, ABI exports,
gloo multi-process tests).
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "clad-3dgs_b200"
for path in (ROOT, PACKAGE, ROOT / "oracle"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
