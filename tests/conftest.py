"""Shared fixtures.  Tests that need a GPU are marked ``gpu``; everything
else runs on the CPU (the oracle, the host logic, the repack arithmetic, and
the C-ABI library's exports)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session", autouse=True)
def _native_built():
    from dotnetfoundryllm_b200 import build
    from oracle import oracle
    build.build()
    oracle.build()


_IMAGES: dict = {}


def model_image(name: str) -> np.ndarray:
    """Seeded synthetic GGUF image (cached per test session)."""
    if name not in _IMAGES:
        from dotnetfoundryllm_b200 import ggufgen
        _IMAGES[name] = ggufgen.build_model(name)
    return _IMAGES[name]


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
