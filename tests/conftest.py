import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_B1H2S544D64.pt")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden():
    import torch
    return torch.load(GOLDEN)


@pytest.fixture(scope="session")
def lib():
    from chia_proj_b200 import build
    build.build()
    from chia_proj_b200 import _native
    return _native.load()


@pytest.fixture(scope="session")
def cuda():
    """The GPU tests run only on a B200 box; fail loudly elsewhere."""
    import torch
    assert torch.cuda.is_available(), "gpu-marked test needs CUDA"
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "needs an sm_100 (B200) device"
    return torch.device("cuda", 0)
