import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def gdn():
    """The product package (directory track-c-gdn_b200/)."""
    return importlib.import_module("track-c-gdn_b200")


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"
