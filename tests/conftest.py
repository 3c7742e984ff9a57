"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` tests run on a CPU-only box (oracle pins, host-side argument
checks, C-ABI symbol exports).  ``-m gpu`` tests need a CUDA device and call
the CUDA path through the C-ABI / torch ops.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "gdn-recoverssm-ascend_b200"
for p in (str(ROOT), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cuda_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
