import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mimizuku_b200 as m
    m.init(0)
    return torch


@pytest.fixture(scope="session")
def ref(cuda):
    from _oracle import REF_FATBIN, RefKernels
    if not os.path.exists(REF_FATBIN):
        pytest.fail(f"{REF_FATBIN} is missing: build it with `make -C oracle ref` (where the reference is present)")
    return RefKernels()
