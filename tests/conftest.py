"""Shared pytest setup: the ``gpu`` marker and import paths for the package and oracle."""

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "bridge-aware-kv-cache-eviction-for-efficient-long-context-transformers_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir():
    return REPO / "tests" / "golden"
