import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libfam.so")


@pytest.fixture(scope="session")
def fam():
    """The product package (directory name is not an identifier)."""
    return importlib.import_module("faster-action-models_b200")


@pytest.fixture(scope="session")
def fam_ops():
    return importlib.import_module("faster-action-models_b200.ops")
