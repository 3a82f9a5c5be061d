"""Test configuration: import paths and the `gpu` marker.

CPU tests (``-m "not gpu"``) check the oracle against the reference's own
known-answer vectors and golden fixtures, the host-side logic, and that the
C-ABI library loads and exports every declared symbol.  GPU tests (``-m gpu``)
compare the CUDA path, called through the C ABI, with the oracle.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "gguf-reader_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA path)")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def ggc():
    import gguf_cuda
    gguf_cuda.lib()
    return gguf_cuda


@pytest.fixture(scope="session")
def ctx(ggc):
    c = ggc.default_context()
    yield c
