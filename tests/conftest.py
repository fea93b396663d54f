"""pytest configuration: import paths and the ``gpu`` marker.

Tests marked ``gpu`` need an sm_100 GPU and the built ``libfqkv.so``; everything else
runs on the CPU.  When no GPU is visible the ``gpu`` tests are skipped (the driver
selects them with ``-m gpu`` on a GPU box, where a missing library fails loudly).
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "fused-triton-rmsnorm-residual-qkv_b200"
for p in (str(PKG_ROOT), str(ROOT), str(Path(__file__).resolve().parent / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
