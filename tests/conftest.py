"""Shared fixtures.  Tests marked `gpu` need a B200; everything else runs on CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build

    build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available

    if not reference_available():
        pytest.skip("oracle/_ref (the reference build) is not present")
    return Reference()


@pytest.fixture(scope="session")
def lib():
    """The product library (libcllm_cuda.so); built in-tree if missing."""
    from cllm_inference_b200 import _lib, build

    build.build()
    return _lib.load()


@pytest.fixture(scope="session")
def cuda(lib):
    """A CUDA device with the library initialised on it; fails (not skips) without one."""
    import torch

    assert torch.cuda.is_available(), "gpu-marked test needs a CUDA device"
    torch.cuda.init()
    from cllm_inference_b200 import _lib

    _lib.check(lib.cllm_cuda_init(0))
    return torch.device("cuda:0")
