import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


@pytest.fixture(scope="session")
def rb():
    """The product library, built in-tree if needed; GPU tests only."""
    import torch
    import remora_b200
    from remora_b200 import build

    build.build()
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return remora_b200


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.lib()
    return oracle
