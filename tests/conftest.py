"""Pytest configuration for the tvarant B200 backend.

``-m "not gpu"`` runs everywhere (oracle pins, host logic, symbol exports,
compiler passes, gloo multi-rank logic).  ``-m gpu`` needs a CUDA device and
the built libraries; those tests are the parity tests proper.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libraries")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def rel_frobenius(y, ref) -> float:
    """||y - ref||_F / ||ref||_F in float64."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref.ravel())
    num = np.linalg.norm((y - ref).ravel())
    return float(num / den) if den > 0 else float(num)


def max_rel(y, ref, floor: float = 1e-30) -> float:
    """max |y - ref| / max(|ref|, floor) elementwise."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref) / np.maximum(np.abs(ref), floor))) if ref.size else 0.0


@pytest.fixture(scope="session")
def rng():
    return np.random.default_rng(1234)
