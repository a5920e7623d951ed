"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``);
* puts the package directory and the oracle on ``sys.path``;
* exposes the golden fixtures generated from the reference kernels.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "diffusion-profiled_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden" / "reference_kernels.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    import fp8_b200  # noqa: F401  (loads libfp8ops.so; fails loudly if missing)

    return torch.device("cuda", 0)
