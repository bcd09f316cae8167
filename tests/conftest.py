"""Shared fixtures.  Tests marked `gpu` need a CUDA device (a B200); everything
else runs on the CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu)")


@pytest.fixture(scope="session")
def golden():
    def load(name: str):
        return dict(np.load(GOLDEN / f"{name}.npz"))
    return load


@pytest.fixture(scope="session")
def ext():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test needs CUDA")
    from cugo_b200 import load_extension
    return load_extension()


@pytest.fixture(scope="session")
def oracle():
    from oracle import ref
    if not ref.available():
        from oracle import build as oracle_build
        oracle_build.build()
    return ref
