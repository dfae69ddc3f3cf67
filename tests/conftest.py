import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_cases(name: str) -> dict:
    """golden/<name>.npz -> {case: {field: array}}."""
    data = np.load(GOLDEN / f"{name}.npz")
    cases: dict = {}
    for key in data.files:
        case, field = key.split("__", 1)
        cases.setdefault(case, {})[field] = data[key]
    return cases


@pytest.fixture(scope="session")
def prescan_golden():
    return load_cases("prescan")


@pytest.fixture(scope="session")
def conv_golden():
    return load_cases("conv")


@pytest.fixture(scope="session")
def lif_golden():
    return load_cases("lif")
