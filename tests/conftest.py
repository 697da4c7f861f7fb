"""Shared pytest setup: import paths, the `gpu` marker, a per-test seeded generator, and a build
of the extension when it is missing (it is git-ignored, so a fresh checkout has none).

GPU tests are marked `gpu` and skipped when no CUDA device is visible (the reference's
conftest.py:10-17 does the same). Everything else runs on the CPU: the oracle against the
golden vectors, the host logic, and that the C-ABI library loads and exports every symbol
include/spectral_b200.h declares.
"""

from __future__ import annotations

import shutil
import sys
import zlib
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "gpu-spectral-stack_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def _ensure_built() -> None:
    lib = PKG / "spectral" / "libspectral_b200.so"
    shims = list((PKG / "spectral").glob("_C*.so"))
    if lib.exists() and shims:
        return
    if shutil.which("nvcc") is None:
        return  # the import below will fail with a message that says how to build
    sys.path.insert(0, str(PKG))
    import build  # gpu-spectral-stack_b200/build.py

    build.build()


_ensure_built()

import torch  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; skipped when none is visible")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def no_device_faults(request):
    """After every GPU test: no kernel may have given up on a bounded wait (tma.cuh)."""
    yield
    if "gpu" in request.node.keywords and torch.cuda.is_available():
        from spectral import native

        torch.cuda.synchronize()
        assert native.device_faults(clear=True) == 0, "a kernel recorded a wait timeout"


@pytest.fixture
def rng(request) -> np.random.Generator:
    """Seeded from the test's id: every case draws the same numbers in any order."""
    return np.random.default_rng(zlib.crc32(request.node.nodeid.encode()))
