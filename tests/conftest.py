import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA libraries")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tinytrain_b200 import _ttk
    _ttk.call("ttk_init", torch.cuda.current_device())
    return torch.device("cuda", torch.cuda.current_device())


@pytest.fixture(scope="session")
def golden_ops():
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "ops_small.npz")))


def rel_err(a, b):
    """max |a - b| / max |b|: the normalised max error used throughout."""
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = max(float(np.abs(b).max()), 1e-30)
    return float(np.abs(a - b).max()) / den
