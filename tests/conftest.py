import os
import sys

import pytest

# cuBLAS is deterministic only with a fixed workspace; it must be set before
# the first cuBLAS handle exists (the end-to-end training test needs it)
os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda", 0)
