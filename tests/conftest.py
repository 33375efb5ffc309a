import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mlx-bun_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built libkvq.so")


@pytest.fixture(scope="session")
def golden_rotating():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "rotating_kvq_mechanics.npz")))
