import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built kernel library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False)
    d = {k: z[k] for k in z.files}
    d["arch"] = json.loads(str(d["arch"]))
    d["dtype"] = str(d["dtype"])
    return d


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from awesome_acceleration_b200 import _lib
    _lib.load()
    return torch.device("cuda")
