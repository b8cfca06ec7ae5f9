"""pytest configuration: registers the `gpu` marker and loads the package by path."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__ as ge

    mod = ge.load_package()
    mod.ensure_custom_op_registered()
    return mod


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    return torch.device("cuda", 0)
