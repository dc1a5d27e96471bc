"""Shared pytest set-up.

Markers:
  gpu -- needs a CUDA device (a B200); skipped when none is visible.  These are
         the parity tests proper: they call the kernels through the C ABI and
         compare against the CPU oracle in ``oracle/``.

The unmarked tests run anywhere: the oracle against the golden vectors made by
the reference's own code, the host-side format logic, and the C ABI's symbol
table / argument validation (no kernel launches).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

HAS_CUDA = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a CUDA device (B200)")


def pytest_collection_modifyitems(config, items):
    if HAS_CUDA:
        return
    skip = pytest.mark.skip(reason="no CUDA device available")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


@pytest.fixture(scope="session", autouse=True)
def _exact_fp32_reference():
    if HAS_CUDA:
        torch.backends.cuda.matmul.allow_tf32 = False
    yield


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


def max_rel(y, ref) -> float:
    """The acceptance metric: max|y - ref| / max|ref| (5e-3 gate)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(y - ref).max() / np.abs(ref).max())


def mean_rel(y, ref) -> float:
    """The reference suite's metric: max|y - ref| / mean|ref|."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(y - ref).max() / np.abs(ref).mean())
