"""Shared test setup: import paths, the ``gpu`` marker, in-tree builds."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for sub in ("python-slm_b200", "oracle"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    """Build the oracle and libslmopt.so in tree if missing or stale."""
    import slm_oracle
    from slmopt import build

    if not slm_oracle.LIB_PATH.exists():
        slm_oracle.build()
    if build.is_stale():
        build.build()
    yield


@pytest.fixture(scope="session")
def kats():
    import json

    return json.loads((ROOT / "tests" / "golden" / "reference_kats.json").read_text())["values"]


def have_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False
