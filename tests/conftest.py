"""Shared pytest configuration.

Markers
-------
gpu : needs a CUDA device (the parity tests proper, calling through the C-ABI library).
      Everything unmarked runs on a CPU-only host.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PACKAGE = "rockchip-npu-notes_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200)")


def load_package():
    """Import the product package (its directory name is not a Python identifier)."""
    return importlib.import_module(PACKAGE)


@pytest.fixture(scope="session")
def b2():
    return load_package()


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    return oracle


def have_gpu():
    try:
        return load_package().device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_fd(b2):
    """One opened device handle for the whole GPU session (device 0)."""
    if b2.device_count() < 1:
        pytest.fail("a gpu-marked test ran without a CUDA device")
    fd = b2.open_device(0)
    yield fd
    b2.close(fd)
