import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libaestrix_cuda.so")


@pytest.fixture(scope="session")
def cuda_ctx():
    import torch
    from aestrix_b200 import _lib

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test ran without a CUDA device")
    torch.cuda.init()
    return _lib.context(0)
