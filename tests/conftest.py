import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100)")


@pytest.fixture(scope="session")
def lib():
    """The ffn_b200 C-ABI library (built from source first when out of date)."""
    from ffn_optim_b200 import _lib

    return _lib.load()
