"""Test configuration.

Markers:
  gpu -- needs a CUDA device (B200); run with `pytest -m gpu`.  Everything
         else runs on the CPU (`pytest -m "not gpu"`).
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA (sm_100a) device")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def oracle_lib():
    """ctypes handle of the C oracle (oracle/_build/libnm_oracle.so), built on demand."""
    import ctypes
    import subprocess

    so = ROOT / "oracle" / "_build" / "libnm_oracle.so"
    if not so.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)
    lib = ctypes.CDLL(str(so))
    P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    lib.nm_gemv_ref.argtypes = [P, P, P, P, I64, I64, I64, I32, I32, I32]
    lib.nm_gemv_ref.restype = None
    return lib
