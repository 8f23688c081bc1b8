import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mlxfast-challenge_senpai_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) >= (10, 0), f"needs sm_100, got sm_{major}{minor}"
    import b2moe

    b2moe.lib()
    return torch.device("cuda", 0)
