"""Test configuration: the ``gpu`` marker, import paths and shared fixtures.

``pytest -m "not gpu"`` runs the CPU suite (oracle vs golden vectors, host logic,
C-ABI load/exports, gloo multi-process); ``pytest -m gpu`` runs the parity
tests on a B200 through the C ABI.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "specdec-context-scaling_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden" / "golden_v1.pt"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import torch

    return torch.load(GOLDEN, weights_only=False)


@pytest.fixture(scope="session")
def lib():
    from specdec_b200 import _lib

    return _lib.load_library()
