"""Shared fixtures: repository on sys.path, the `gpu` marker, golden corpus."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libglq.so")


@pytest.fixture(scope="session")
def golden():
    """(arrays, manifest) of tests/golden/corpus.npz + manifest.json."""
    arrays = dict(np.load(GOLDEN / "corpus.npz"))
    manifest = json.loads((GOLDEN / "manifest.json").read_text())
    return arrays, manifest


def f16(arr: np.ndarray) -> np.ndarray:
    """uint16 fixture bits -> float16 array."""
    return arr.view(np.float16)


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for -m gpu tests (no silent skip)")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"sm_100a kernels need compute capability 10.0, found {major}.{minor}")
    return torch.device("cuda", 0)
