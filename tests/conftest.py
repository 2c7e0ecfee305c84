"""Shared pytest configuration: the ``gpu`` marker and golden-fixture loaders."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def golden_arrays():
    with np.load(GOLDEN_DIR / "golden.npz") as data:
        return {key: data[key] for key in data.files}


@pytest.fixture(scope="session")
def golden_meta():
    return json.loads((GOLDEN_DIR / "golden.json").read_text())


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test is marked gpu and needs a CUDA device (B200, sm_100a)")
    return torch.device("cuda", torch.cuda.current_device())
