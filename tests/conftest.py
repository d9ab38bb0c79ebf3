"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200) and the in-tree sm_100a
library; everything else runs on CPU.  The oracle under ``oracle/`` is the
checker in both cases.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the sm_100a library")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return torch.device("cuda:0")
