import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))
GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running parity case")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def host_golden(golden_dir):
    """Host-logic fixtures recorded from the reference's own modules."""
    import json

    return json.loads((golden_dir / "host_logic.json").read_text())


@pytest.fixture(scope="session")
def lib():
    from superl8_serve_b200 import _lib

    return _lib.load()


def pytest_sessionstart(session):
    os.environ.setdefault("S8B_TEST", "1")
