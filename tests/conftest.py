"""Shared pytest setup.

* Registers the ``gpu`` marker: tests that need a CUDA device (B200, sm_100a).
* Puts the repo root (for ``oracle``) and ``solution-is-all-you-need_b200``
  (for the ``phantom_moe`` package) on ``sys.path``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "solution-is-all-you-need_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import phantom_moe
    phantom_moe.load_library()  # raises if the library is missing: no silent fallback
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _clear_device_error(request):
    """The library's device error word (phmoe_device_error) accumulates until
    it is read with reset; clear it before each GPU test so a test that checks
    it sees only what its own calls raised."""
    if request.node.get_closest_marker("gpu") is not None:
        import torch
        if torch.cuda.is_available():
            import phantom_moe
            phantom_moe.load_library().phmoe_device_error(1)
    yield
