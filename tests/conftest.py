"""Shared pytest configuration.

Markers: ``gpu`` -- needs a CUDA device (B200, sm_100a); run with ``-m gpu``.
CPU tests (``-m "not gpu"``) cover the oracle against the golden fixtures, the
host logic and the C-ABI library's exports and argument checks.
"""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_arrays():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="session")
def golden_meta():
    return json.loads((GOLDEN / "golden.json").read_text())
