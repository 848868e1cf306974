"""Shared pytest configuration.

Tests that need a B200 are marked ``gpu``; the CPU suite is
``pytest tests -m "not gpu"`` and the GPU suite ``pytest tests -m gpu``.
"""
import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built extension")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _few_threads():
    old = torch.get_num_threads()
    torch.set_num_threads(min(old, 4))
    yield
    torch.set_num_threads(old)


@pytest.fixture
def native():
    """The loaded extension (GPU tests fail, not skip, when it is missing)."""
    from exploration_b200.ops import _native
    return _native.load(required=True)


os.environ.setdefault("EB200_PG_TIMEOUT_S", "60")
