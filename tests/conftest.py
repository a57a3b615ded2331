"""pytest configuration: import paths, the `gpu` marker, shared fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "arc-gemm_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def native_lib():
    """The built libarcb200.so (built here if missing; the build is CPU-only)."""
    from arc import build

    build.build()
    from arc._lib import lib

    return lib()


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    from oracle.build import build_oracle

    build_oracle()
