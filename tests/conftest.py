"""Shared fixtures.  `-m gpu` tests need a B200; everything else runs on CPU."""
from __future__ import annotations

import shutil
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def _ensure_library() -> Path:
    from oct_b200 import build
    lib = build.LIB_PATH
    if not lib.exists() or (shutil.which("nvcc") or Path("/usr/local/cuda/bin/nvcc").exists()):
        # Rebuild when sources changed and a toolchain is present; on a machine
        # without nvcc the prebuilt in-tree library is used as is.
        try:
            build.build_library()
        except Exception:
            if not lib.exists():
                raise
    return lib


@pytest.fixture(scope="session")
def lib():
    _ensure_library()
    from oct_b200.reactor import load_library
    return load_library()


@pytest.fixture(scope="session")
def golden():
    return np.load(REPO / "tests" / "golden" / "known_answers.npz")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def runtime(lib):
    from oct_b200.reactor import Runtime
    rt = Runtime(lib)
    yield rt
    rt.close()
