"""Shared pytest configuration: the ``gpu`` marker and build fixtures."""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def built_lib():
    """Path of libbag_b200.so, building it first when it is missing or stale."""
    from bag_b200 import build
    return build.build()


@pytest.fixture(scope="session")
def bag(built_lib):
    import bag_b200
    bag_b200.lib()
    return bag_b200


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    return torch.device("cuda:0")
