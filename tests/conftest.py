"""Shared test fixtures.

``-m gpu`` tests need a B200 and the built library; everything else runs on
the CPU (oracle pins, host logic, C-ABI loading, gloo multi-rank tests).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and libdflash_b200.so")


@pytest.fixture(scope="session")
def pkg():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def to_dev_bf16(a: np.ndarray, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)


def to_dev_u32(a: np.ndarray, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(dev)


def bf16_to_np_bits(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
