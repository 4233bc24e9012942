"""Shared test setup.  GPU tests are marked ``gpu`` and run only on a B200
(``pytest -m gpu``); everything else runs on a CPU-only machine."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))

GOLDEN = Path(__file__).resolve().parent / "golden" / "kats.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def kats():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def device():
    import zengpu_b200 as zg
    if zg.device_count() == 0:
        pytest.fail("GPU test collected but no CUDA device is visible")
    dev = zg.CudaDevice(0)
    yield dev
    dev.close()


@pytest.fixture(scope="session")
def pool(device):
    import zengpu_b200 as zg
    p = zg.BufferPool(device)
    yield p
    p.close()
