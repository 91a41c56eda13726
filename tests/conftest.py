"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; on a machine without a
CUDA device they are skipped, on a GPU box they run against the in-tree
libtinygiant.so (which must exist: no fallback)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libtinygiant.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def _has_gpu() -> bool:
    try:
        from tinygiant_b200._lib import load_tinygiant_lib
        lib = load_tinygiant_lib()
        return bool(lib) and lib.tg_device_count() > 0
    except OSError:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(ROOT / "tests" / "golden" / "golden_q4_0.npz"))


@pytest.fixture(scope="session")
def lib():
    from tinygiant_b200._lib import get_lib
    return get_lib()
