"""Shared test setup: the `gpu` marker, the oracle build and fixture paths.

`-m "not gpu"` tests run on the CPU (oracle vs golden vectors, host logic,
library exports); `-m gpu` tests drive libsrstep.so on a B200 through its C ABI
and compare with the oracle.
"""

import glob
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
GOLDEN = sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libsrstep.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def srlib():
    """The built product library; GPU tests fail loudly if it is missing."""
    from sr_go_tranformer_b200 import build as B
    B.build()
    from sr_go_tranformer_b200 import _abi
    return _abi.lib()
