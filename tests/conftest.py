"""Shared pytest setup: import paths, the ``gpu`` marker and GPU fixtures."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "multi-lora-llm-kernel_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden" / "golden_bgmv.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    return torch.device("cuda", 0)
