"""Shared test setup: the ``gpu`` marker, library builds and helpers.

CPU-only tests (``-m "not gpu"``) build the product library with nvcc (cross
compilation, no GPU needed) and the C oracle with gcc. GPU tests call the
library through its C ABI (kvbridge_b200.api -> libkvbridge_b200.so).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def kvb_lib():
    from kvbridge_b200 import build

    build.build()
    from kvbridge_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build(ref=oracle.REFERENCE_DIR.exists() and not oracle.REF_ORACLE_LIB.exists())
    return oracle


@pytest.fixture(scope="session")
def cuda_device(kvb_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("kernels are built for sm_100a only")
    torch.cuda.init()
    return torch.device("cuda:0")
