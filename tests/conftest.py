from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str):
    return np.load(GOLDEN / f"{name}.npz", allow_pickle=False)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> exact float32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def cfg1_inputs():
    """BASELINE config 1 (seed 0): q ~ N(0,1)/sqrt(128), w ~ N(0,1)/sqrt(64), K ~ N(0,1)."""
    import torch

    g = torch.Generator().manual_seed(0)
    q = torch.randn(64, 128, generator=g) / math.sqrt(128)
    w = torch.randn(64, generator=g) / math.sqrt(64)
    k = torch.randn(4096, 128, generator=g)
    return q, w, k


@pytest.fixture(scope="session")
def golden():
    return load_golden
