"""Shared test setup: the ``gpu`` marker, import paths, fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def kat():
    """Known-answer fixtures from tests/golden/make_golden.py."""
    data = np.load(ROOT / "tests" / "golden" / "kat.npz")
    cases = {}
    for key in data.files:
        name, rest = key.split("/", 1)
        c = cases.setdefault(name, {"w": {"content_proj_w": None, "content_proj_b": None}})
        if rest.startswith("w/"):
            c["w"][rest[2:]] = data[key]
        else:
            c[rest] = data[key]
    return cases


@pytest.fixture(scope="session")
def ctx():
    """One wave_engine_b200 context on cuda:0 (GPU tests only)."""
    import wave_engine_b200 as wb
    c = wb.Context(0)
    yield c
    c.close()
