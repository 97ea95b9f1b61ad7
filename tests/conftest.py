"""Test configuration: the ``gpu`` marker, import paths and shared fixtures.

``gpu`` tests need a CUDA device (a B200); without one they are skipped. Everything else
runs on the CPU: the oracle against the reference's golden vectors, the host-side logic of
the package and the C-ABI library's exported symbols.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "kernel-agent_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a)")


def _cuda() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    """The reference's golden vectors (``tests/golden/golden.npz``)."""
    with np.load(GOLDEN / "golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_meta():
    """The reference's comparator and scale-check results (``tests/golden/golden.json``)."""
    return json.loads((GOLDEN / "golden.json").read_text())
