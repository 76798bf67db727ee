"""Shared pytest configuration.

Markers: ``gpu`` -- needs a CUDA device (B200) and the built extension.  The
CPU suite (``-m "not gpu"``) covers the oracle against the reference's golden
vectors, the host-side logic and that the C-ABI library loads.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "decode-kernel_b200", REPO / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: full-size BASELINE shapes (tens of seconds)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch.device("cuda", 0)
