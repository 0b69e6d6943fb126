import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built kernel library")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly when selected without a GPU rather than skipping.
    pass


@pytest.fixture(scope="session")
def golden():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "c1_reference.pt", weights_only=False)
