import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "bert-by-hand_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


@pytest.fixture(scope="session")
def golden_unit():
    import numpy as np

    return dict(np.load(os.path.join(ROOT, "tests", "golden", "unit.npz")))


@pytest.fixture(scope="session")
def golden_model():
    import numpy as np

    return dict(np.load(os.path.join(ROOT, "tests", "golden", "model.npz")))
