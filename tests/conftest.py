"""Shared pytest configuration.

Markers: `gpu` for tests that need a CUDA device (run with `-m gpu` on a
B200); everything else runs on the CPU (`-m "not gpu"`).
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def kv():
    import kvflux_b200

    return kvflux_b200


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.lib()
    return o
