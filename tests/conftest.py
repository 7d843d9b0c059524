import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """The oracle (C restatement) is cheap to build; the CUDA library must be
    prebuilt by __graft_entry__.build() or moestream_b200/csrc/build.py."""
    from oracle import oracle
    if not os.path.exists(oracle.LIBORACLE):
        oracle.build()
    yield


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
