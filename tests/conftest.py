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


def pytest_terminal_summary(terminalreporter):
    """Print how far each logged parity check sat from the oracle (max |diff|
    and the fraction of outputs beyond 2e-3), passing or not."""
    try:
        from helpers import PARITY_LOG
    except Exception:
        return
    if not PARITY_LOG:
        return
    terminalreporter.section("parity vs oracle (max |diff|, fraction beyond 2e-3)")
    for name, m, beyond, bar in PARITY_LOG:
        terminalreporter.write_line(f"{name}: max|diff| {m:.3e}, beyond 2e-3 {beyond:.2e} [{bar}]")
