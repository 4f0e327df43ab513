import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "longcat-video-mlx_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built engine library")


@pytest.fixture(scope="session")
def cuda():
    """GPU tests fail (not skip) without a device: a silent skip would hide a missing GPU path."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    from longcat_video import _native

    _native.lib()
    return torch.device("cuda:0")
