import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    """GPU tests fail (not skip) when no CUDA device is present: they are run
    only where a B200 is expected."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"expected sm_100 (B200), got sm_{major}{minor}"
    return torch.device("cuda:0")
