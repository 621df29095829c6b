import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden_weights():
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "glad_weights.npz")))


@pytest.fixture(scope="session")
def golden_fwd():
    import numpy as np
    return {b: dict(np.load(os.path.join(GOLDEN, f"glad_fwd_b{b}.npz"))) for b in (1, 3, 16)}


@pytest.fixture(scope="session")
def golden_conv():
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "glad_conv_b4.npz")))
