"""Shared pytest configuration.

Tests marked ``gpu`` need a B200 and the CUDA library; everything else runs
on the CPU (the driver runs ``pytest -m "not gpu"`` without a GPU).
"""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"
ORACLE_LIB = REPO / "oracle" / "_build" / "libqa_oracle.so"
REF_LIB = REPO / "oracle" / "_ref" / "libqa_kernels_ref.so"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the CUDA library")


def _ensure_oracle():
    if not ORACLE_LIB.exists():
        subprocess.run(["make", "-C", str(REPO / "oracle"), "oracle"], check=True,
                       capture_output=True)
    return ORACLE_LIB


@pytest.fixture(scope="session")
def oracle():
    """The C oracle loaded through the product's ctypes wrapper."""
    from quantanything_b200.native import KernelLibrary

    return KernelLibrary(_ensure_oracle())


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "kernels.npz"))


@pytest.fixture(scope="session")
def gpu_lib():
    """The CUDA library (skips the test when no GPU is present)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from quantanything_b200 import native

    return native.get_library()
