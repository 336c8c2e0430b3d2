"""Test configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs on any host (oracle vs golden vectors, host logic, the
C ABI's exports).  ``-m gpu`` tests call the CUDA library through its C ABI on
a B200 and compare against the oracle; they are skipped only when no CUDA
device exists at all -- a missing library is a failure, not a skip.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str):
    import numpy as np
    return np.load(GOLDEN / f"{name}.npz", allow_pickle=False)


def unpack_lists(data, prefix: str):
    return [list(data[f"{prefix}_{i}"]) for i in range(int(data[f"{prefix}_count"]))]
