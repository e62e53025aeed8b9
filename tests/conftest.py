import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long CPU test")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(REPO / "tests" / "golden" / "golden.npz")


@pytest.fixture(scope="session")
def cache_policy_golden():
    import json

    return json.loads((REPO / "tests" / "golden" / "cache_policy.json").read_text())
