import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


@pytest.fixture(scope="session")
def backend():
    """One B200Backend on cuda:0 for the GPU tests (libfi8_b200.so; no fallback)."""
    from aikit_b200.ann import B200Backend
    return B200Backend(0)
