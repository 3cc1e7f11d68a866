import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG = "3080_mod_p2p_sglang_patch_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


def pkg():
    return importlib.import_module(PKG)


def sub(name):
    return importlib.import_module(f"{PKG}.{name}")


@pytest.fixture(scope="session")
def mbx():
    return pkg()


def free_port():
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p
