import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO / "epic-kernel_b200", REPO, REPO / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libek.so")


@pytest.fixture(scope="session")
def golden_dir():
    return REPO / "tests" / "golden"
