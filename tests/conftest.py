"""Test configuration: import paths and the ``gpu`` marker."""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
PACKAGE_PARENT = os.path.join(ROOT, "hayate-exp_b200")
for path in (ROOT, TESTS, PACKAGE_PARENT):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


def pytest_collection_modifyitems(config, items):
    # GPU tests need a device; on a CPU host they are skipped rather than failed.
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch is part of the image
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
