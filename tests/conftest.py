import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib():
    from da3cpplib_b200 import _lib

    return _lib.load()


def cuda_stream_ptr():
    import torch

    return ctypes_void(torch.cuda.current_stream().cuda_stream)


def ctypes_void(v):
    import ctypes

    return ctypes.c_void_p(v)
