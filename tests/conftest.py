"""Shared pytest setup: the `gpu` marker, import paths for the product package (jkb200) and the
CPU oracle (test infrastructure), and small helpers used by several test files."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_PARENT = os.path.join(ROOT, "jero-kernels-rvv_b200")
for p in (PKG_PARENT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import pyoracle

    pyoracle.lib()
    return pyoracle


@pytest.fixture(scope="session")
def jkb():
    """The product package; GPU tests fail loudly (no skip) if CUDA or the .so is missing."""
    import torch

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    import jkb200

    jkb200.abi_version()
    return jkb200
