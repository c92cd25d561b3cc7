"""Shared test setup.

* `gpu` marks tests that need a CUDA device (run with `-m gpu` on a B200).
* The engine (vd-ttfs_b200/vdttfs + libvdttfs.so) and the CPU oracle
  (oracle/) are put on sys.path; the oracle is the checker, never the thing
  under test.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def O():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def dev():
    if not cuda_ok():
        pytest.fail("GPU test selected but torch.cuda.is_available() is False")
    import torch
    torch.cuda.init()
    return torch.device("cuda:0")
