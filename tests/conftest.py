import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly without a GPU rather than skipping silently, but
    # only when they were selected (`-m gpu`); a plain run deselects nothing.
    pass


@pytest.fixture(scope="session")
def device() -> int:
    return int(os.environ.get("OMG_TEST_DEVICE", "0"))
