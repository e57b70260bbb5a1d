"""pytest configuration: the `gpu` marker, import paths, shared helpers.

Tests marked gpu need a B200 (sm_100) and the built liblfm2q.so; everything else runs on CPU.
"""

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "lfm2.5-vl-optimization_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built liblfm2q.so")


def golden(name):
    return np.load(GOLDEN / f"{name}.npz")


def to_t(a, bf16=False):
    """numpy fixture array -> torch tensor (bf16 arrays are stored as their int16 bit patterns)."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.view(torch.bfloat16) if bf16 else t


@pytest.fixture(scope="session")
def cuda_dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.skip("needs an sm_100 (B200) device")
    return torch.device("cuda", torch.cuda.current_device())
