"""Test configuration: the `gpu` marker selects tests that need a B200."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run on the B200 box)")
    config.addinivalue_line("markers", "slow: full-size (3B) parity; minutes of CPU oracle time")


@pytest.fixture(scope="session")
def golden():
    return GOLDEN
