"""Shared test configuration: the ``gpu`` marker and golden-fixture loaders."""
from __future__ import annotations

import gzip
import json
import math
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libpmb200")


def load_golden(name: str):
    with gzip.open(GOLDEN / name, "rt") as f:
        return json.load(f)


def close(a, b, rel=1e-6, abs_=1e-9) -> bool:
    """Recursive equality with a relative tolerance for floats (NaN equals NaN)."""
    if isinstance(a, bool) or isinstance(b, bool) or a is None or b is None or isinstance(a, str) or isinstance(b, str):
        return a == b
    if isinstance(a, (int, float)) and isinstance(b, (int, float)):
        if isinstance(a, float) and isinstance(b, float) and math.isnan(a) and math.isnan(b):
            return True
        return a == b or abs(a - b) <= max(rel * max(abs(a), abs(b)), abs_)
    if isinstance(a, dict) and isinstance(b, dict):
        return a.keys() == b.keys() and all(close(a[k], b[k], rel, abs_) for k in a)
    if isinstance(a, (list, tuple)) and isinstance(b, (list, tuple)):
        return len(a) == len(b) and all(close(x, y, rel, abs_) for x, y in zip(a, b))
    return a == b


def diff(expected: dict, actual: dict, keys, rel=1e-6) -> list[str]:
    out = []
    for k in keys:
        if k not in expected:
            continue
        if not close(expected[k], actual.get(k), rel):
            out.append(f"{k}: expected {expected[k]!r} got {actual.get(k)!r}")
    return out


@pytest.fixture(scope="session")
def gpu_ready():
    from powermodeling_b200 import _native as N
    if N.library().pm_device_count() < 1:
        pytest.fail("GPU test ran without a visible CUDA device")
    return N
