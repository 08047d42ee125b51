import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the oracle and the native libraries once per session (nvcc cross-compiles)."""
    from oracle import pxo
    pxo.build()
    from proxima_b200 import build
    build.build_all()
    yield
