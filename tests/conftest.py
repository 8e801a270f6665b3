"""Shared pytest setup: import paths, the `gpu` marker, and fixtures for the oracle libraries."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "train.cpp_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def ref():
    import oracle

    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libtrc_ref.so not built (needs the train.cpp sources)")
    return oracle


@pytest.fixture(scope="session")
def goldens():
    return {
        "reference": np.load(GOLDEN / "reference_goldens.npz"),
        "dequant": np.load(GOLDEN / "dequant_goldens.npz"),
        "mul_mat": np.load(GOLDEN / "mul_mat_goldens.npz"),
    }


def normwise(got: np.ndarray, want: np.ndarray) -> float:
    """max|got - want| / max|want| (the accuracy metric of the mul_mat path)."""
    den = float(np.max(np.abs(want))) if want.size else 0.0
    num = float(np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)))) if want.size else 0.0
    return num / den if den > 0 else num
