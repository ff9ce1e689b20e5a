"""Shared pytest setup: markers, repo paths and helpers."""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "logic-bs-roformer-rs_b200"
for p in (REPO, PKG, REPO / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU oracle work")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(REPO / "tests" / "golden" / "dump_refs_subset.npz")


@pytest.fixture(scope="session")
def demix_golden():
    import numpy as np
    return np.load(REPO / "tests" / "golden" / "demix_identity.npz")
