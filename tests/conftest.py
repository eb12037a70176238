"""Shared pytest setup: the `gpu` marker and fixtures.

Tests marked `gpu` need a B200 (sm_100a) and call the CUDA path through the
C ABI; everything else runs on a CPU-only host.  GPU tests do not skip when
CUDA is missing: on a GPU box a missing device or library is a failure.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built libm1moe_cuda.so")


@pytest.fixture(scope="session")
def golden():
    def load(name: str):
        return dict(np.load(GOLDEN / f"{name}.npz"))
    return load


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


def rel_max_err(y, y_ref) -> float:
    """max |y - y_ref| / ||y_ref||_2 — the tolerance metric of the parity bar."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    return float(np.max(np.abs(y - y_ref)) / max(np.linalg.norm(y_ref), 1e-30))
