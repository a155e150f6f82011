import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture
def golden():
    return load_golden


@pytest.fixture
def cuda():
    """cuda:0 with the library loaded; after the test, no kernel may have left a
    timed-out wait in the device error word (a wait that ran out means some
    kernel returned early, so the test's results cannot be trusted)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mk_iii_technologies_tsrn_b200 import _lib, ops

    _lib.load()  # fails loudly if the library is missing
    dev = torch.device("cuda:0")
    ops.check_device_error(dev)   # start clean
    yield dev
    ops.check_device_error(dev)
