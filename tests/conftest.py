import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


def gpu_count() -> int:
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.fixture(scope="session")
def golden():
    """The fixtures tests/golden/make_golden.py recorded from the reference connector."""
    import json

    import numpy as np

    here = os.path.join(ROOT, "tests", "golden")
    with open(os.path.join(here, "kv_transfer_golden.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(here, "kv_transfer_small.npz")))
    return meta, arrays
