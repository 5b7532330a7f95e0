"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 and the compiled extension; everything else
runs on CPU (multi-process tests use the gloo backend on 127.0.0.1).
"""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

torch.set_num_threads(max(1, min(4, os.cpu_count() or 1)))


def free_port() -> int:
    """A TCP port on 127.0.0.1 that is free right now (for multi-process rendezvous)."""
    import socket

    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the compiled sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def cuda():
    return torch.device("cuda", 0)
