import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "gat-tfs_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels through the C-ABI)")
    config.addinivalue_line("markers", "slow: larger configurations (seconds to minutes)")


@pytest.fixture(scope="session")
def root():
    return ROOT


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def dev():
    """CUDA device for the gpu tests; they fail (not skip) without one."""
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.init()
    return torch.device("cuda:0")
