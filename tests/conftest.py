"""Test setup: import paths, the ``gpu`` marker and the in-tree library build.

``-m "not gpu"`` runs everywhere (oracle vs golden fixtures, host logic, C-ABI
exports); ``-m gpu`` needs a B200 and compares the CUDA path with the oracle.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "disk-mem-off_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU (B200)")


@pytest.fixture(scope="session")
def built_lib() -> str:
    from moe_sm100.build import build
    return build()
