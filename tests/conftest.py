"""Shared pytest configuration.

* registers the ``gpu`` and ``slow`` markers;
* puts the repository root (for ``oracle``) and the package directory (for
  ``lightning_router``) on ``sys.path``;
* ``golden(name)`` loads a committed fixture from ``tests/golden``.
"""

from __future__ import annotations

import functools
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "llm-serving-kernel-optimization_b200"
for p in (str(ROOT), str(PKG_DIR), str(Path(__file__).resolve().parent)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running")


@functools.lru_cache(maxsize=None)
def golden(name: str):
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def lr_ops():
    """The compiled extension; a GPU test fails (not skips) when it is missing."""
    import lightning_router._ext as ext
    return ext.ops()


os.environ.setdefault("PYTHONHASHSEED", "0")
