"""Shared pytest configuration: the ``gpu`` marker gates every device test."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the native extension")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        have_cuda = torch.cuda.is_available()
        n_dev = torch.cuda.device_count() if have_cuda else 0
    except Exception:  # pragma: no cover - torch missing
        have_cuda, n_dev = False, 0
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    skip_multi = pytest.mark.skip(reason="needs >= 2 CUDA devices")
    for item in items:
        if "gpu" in item.keywords and not have_cuda:
            item.add_marker(skip_gpu)
        if "multigpu" in item.keywords and n_dev < 2:
            item.add_marker(skip_multi)
