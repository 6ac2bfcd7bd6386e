"""Shared pytest configuration.

`gpu` marks tests that need a B200 (sm_100a) and the built CUDA library; the CPU suite runs with
`-m "not gpu"`.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU and the CUDA library")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    major, minor = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip(f"sm_100a required, found sm_{major}{minor}")
    return torch.device("cuda", torch.cuda.current_device())
