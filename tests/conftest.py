import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.join(ROOT, "tests")
for _p in (ROOT, TESTS):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_codecs():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "codecs.npz")))


@pytest.fixture(scope="session")
def golden_layers():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "layers.npz")))
