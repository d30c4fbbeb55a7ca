"""Shared test configuration.

Tests marked ``gpu`` need a CUDA device (a B200) and the built native libraries; the
rest run on the CPU. The package lives in ``torch-convnd_b200/`` and the oracle in
``oracle/``; both are put on sys.path here.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
for path in (ROOT / "torch-convnd_b200", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the native build")
    os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    """Loader of the reference-generated golden fixtures."""

    def load(name):
        return torch.load(GOLDEN / f"{name}.pt", weights_only=False)

    return load


@pytest.fixture(scope="session", autouse=True)
def _precision_policy():
    previous = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    threads = torch.get_num_threads()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = previous
        torch.set_num_threads(threads)
