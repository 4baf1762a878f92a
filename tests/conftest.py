"""Test configuration: the ``gpu`` marker, shared fixtures and import paths.

``-m "not gpu"`` runs on any host (oracle, host logic, C-ABI loading and validation);
``-m gpu`` needs a CUDA device and exercises the sm_100a kernels through the public API and the
C ABI.  GPU tests skip (rather than fail) only when no CUDA device is visible at all.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
