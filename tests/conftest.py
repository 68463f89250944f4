"""Shared fixtures.  GPU tests are marked ``@pytest.mark.gpu``; everything else
runs on the CPU (``pytest -m "not gpu"``)."""
import json
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def to_torch(a: np.ndarray, dtype: str) -> torch.Tensor:
    """Golden arrays store bf16/fp16 as uint16 bit patterns."""
    if dtype in ("bfloat16", "float16"):
        return torch.from_numpy(a.view(np.int16).copy()).view(getattr(torch, dtype))
    return torch.from_numpy(a.copy())


@pytest.fixture(scope="session")
def golden_index():
    with open(os.path.join(GOLDEN, "index.json")) as f:
        return json.load(f)


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
