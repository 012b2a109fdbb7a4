import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


@pytest.fixture(scope="session")
def ctx():
    import torch
    import shoehorn_b200 as sh
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = sh.Context(0)
    yield c
    c.close()
