import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the device path against the oracle")
    config.addinivalue_line("markers", "slow: full-size parity run")


@pytest.fixture(scope="session")
def ref():
    from oracle import ref as r

    if not r.available():
        pytest.skip("reference oracle not built (make -C oracle)")
    return r
