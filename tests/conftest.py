import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "integration: exercises several subsystems together")
    config.addinivalue_line("markers", "slow: takes noticeably longer than a unit test")


@pytest.fixture
def cuda_ext():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from wavelet_b200.ops import _ext

    return _ext.load()
