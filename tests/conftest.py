import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "array-morphisms_b200", ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")
    config.addinivalue_line("markers", "slow: full-size workload")


@pytest.fixture(scope="session")
def amc():
    """The product package with its device initialised."""
    import amcuda
    amcuda.init(0)
    return amcuda
