import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def golden():
    path = os.path.join(HERE, "golden", "golden.npz")
    data = np.load(path)
    import json
    with open(os.path.join(HERE, "golden", "manifest.json")) as f:
        manifest = json.load(f)
    return data, manifest


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests.  The native library must be present
    and load: a GPU test never falls back to anything else."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import leap_b200
    from leap_b200 import _native
    _native.lib()  # raises if the sm_100a library is missing
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"expected sm_100 (B200), got sm_{major}{minor}"
    return torch.device("cuda:0")
