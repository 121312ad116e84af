"""Shared fixtures.  ``-m gpu`` tests need a B200; the rest run on CPU."""
from __future__ import annotations

import importlib
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


def load_pkg():
    return importlib.import_module("mini-sglang-fork_b200")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    from oracle import w8a8_oracle

    return w8a8_oracle


@pytest.fixture(scope="session")
def cuda_dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def golden(name: str):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)
