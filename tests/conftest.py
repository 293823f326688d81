"""Shared test setup: the `gpu` marker, the repository on sys.path, and the library / oracle fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def port():
    from oracle.oracle import port as _port

    return _port()


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    d = ROOT / "tests" / "golden"
    return {p.stem: dict(np.load(p)) for p in sorted(d.glob("*.npz"))}


@pytest.fixture(scope="session")
def vox():
    """The vox_b200 package on a CUDA device; built for sm_100a first if the library is missing."""
    import torch

    from vox_b200 import build as _build

    if not _build.LIB.exists():
        _build.build()
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for the gpu tests")
    import vox_b200

    return vox_b200


@pytest.fixture(scope="session")
def vox_lib():
    """The vox_b200 package for host-only calls (the .tmod reader): built if missing, no CUDA device needed."""
    from vox_b200 import build as _build

    if not _build.LIB.exists():
        _build.build()
    import vox_b200

    return vox_b200
