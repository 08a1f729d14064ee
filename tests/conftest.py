"""pytest set-up: the `gpu` marker, import paths, and the native libraries.

`-m "not gpu"` runs everything that needs no GPU (oracle vs golden fixtures, host logic, the C-ABI
library's exports and argument checks, gloo multi-rank harness tests). `-m gpu` runs the parity
tests of the CUDA kernels against the oracle; they fail (not skip) without a CUDA device.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
TESTS = Path(__file__).resolve().parent
for p in (str(ROOT), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (the B200 parity tests)")


@pytest.fixture(scope="session", autouse=True)
def _native_libs():
    """Builds libmas_b200.so (nvcc) and the oracle's liborc.so (gcc) when they are missing or stale."""
    import importlib.util

    # build.py is loaded by path: importing the package would first try to load the library.
    spec = importlib.util.spec_from_file_location("_mas_build", ROOT / "mini-agent-serve_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    import oracle

    oracle.build()
    yield


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)
