"""Shared test setup: import paths, the ``gpu`` marker and golden-fixture access."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "moss-tts-optimized_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long CPU oracle runs")


def golden(name: str):
    return np.load(GOLDEN / f"{name}.npz")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"expected sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda", 0)


def pytest_collection_modifyitems(config, items):
    # Keep the whole CPU suite to a few minutes: the oracle is threaded numpy.
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
