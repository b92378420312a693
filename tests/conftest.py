"""Shared test setup: the `gpu` marker, an in-tree build of the library, and
the oracle build.  CPU tests (`-m "not gpu"`) never launch a kernel."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    from mitten_b200 import _lib, build

    if not _lib.LIB_PATH.exists():
        build.build()
    import oracle

    oracle.build()
    yield


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
