"""Shared test setup: import paths, the `gpu` marker, fixtures.

CPU tests (-m "not gpu") cover the oracle against golden vectors, the host
logic and the C-ABI library's exports.  GPU tests (-m gpu) are the parity
tests proper: they call libvfr_retrieval.so through its C ABI and compare with
the oracle (oracle/) on the same seeded inputs.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "vocal-fast-rs_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests through the C ABI")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o


@pytest.fixture(scope="session")
def native():
    """The built CUDA library (build it first with vocal-fast-rs_b200/build.py)."""
    from vfr import lib

    return lib.load_library()


def golden(name: str) -> bytes:
    with open(os.path.join(GOLDEN, name), "rb") as f:
        return f.read()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch
