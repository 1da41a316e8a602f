"""Shared fixtures.  GPU tests are marked ``gpu`` and call the CUDA backend
through its C ABI (libqsml_cuda.so) via quasarml_b200.abi; the CPU oracle
(oracle/) is the checker."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def orc():
    from oracle import qsml_oracle
    qsml_oracle.lib()
    return qsml_oracle


@pytest.fixture(scope="session")
def ctx():
    import torch
    from quasarml_b200 import abi
    torch.cuda.set_device(0)
    c = abi.Context(0)
    yield c
    torch.cuda.synchronize()
    c.close()
