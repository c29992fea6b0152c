"""Shared test setup: import paths, the ``gpu`` marker and common fixtures.

CPU tests (``-m "not gpu"``) check the oracle against HF transformers and the golden
vectors, the host-side layout / sharding logic, and that the C-ABI library loads and
exports every declared symbol.  GPU tests (``-m gpu``) run the CUDA path through the
C ABI and compare it with the oracle.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "kaggle-tpu-inference_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
