"""Shared fixtures. ``-m gpu`` tests need a CUDA device and call the product
library through its C ABI; everything else runs on the CPU."""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); calls libwhistle_b200.so")


@pytest.fixture(scope="session")
def orc():
    """The CPU oracle (test infrastructure)."""
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def wb():
    """The product package, with its CUDA library built in-tree."""
    mod = importlib.import_module("go-whistle_b200")
    mod.build()
    return mod


@pytest.fixture(scope="session")
def cuda(wb):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a -m gpu test ran without a CUDA device")
    torch.cuda.init()
    return torch
