"""Test configuration: the ``gpu`` marker and import paths.

CPU tests (``-m "not gpu"``) pin the oracle to the golden fixtures and check the
host-side logic and the C-ABI library's exports. GPU tests (``-m gpu``) run the
CUDA kernels through the C-ABI and compare them with the oracle.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_ROOT = ROOT / "faquant-public_b200"
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, PACKAGE_ROOT, GOLDEN):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {key: data[key] for key in data.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden


os.environ.setdefault("PYTHONHASHSEED", "0")
