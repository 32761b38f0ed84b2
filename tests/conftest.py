import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "cutile-triton_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: full BASELINE-size case")


@pytest.fixture(scope="session")
def dev():
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    import cutile_b200

    cutile_b200.ops.init(0)
    return torch.device("cuda:0")
