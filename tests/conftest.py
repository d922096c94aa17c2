"""Shared test setup: import paths, the `gpu` marker, and build-on-demand of
the CPU oracle (test infrastructure) and of the CUDA library."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "pulsar-asm_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    if not os.path.exists(O.LIB_PATH):
        subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle")])
    O.lib()
    return O


@pytest.fixture(scope="session")
def pb():
    import pulsar_b200 as P
    if not os.path.exists(P.LIB_PATH):
        P.build()
    P.lib()
    return P


@pytest.fixture(scope="session")
def cuda(pb):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device")
    torch.cuda.init()
    return torch
