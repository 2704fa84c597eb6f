"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU.

The oracle under oracle/ is the checker here and only here (plus
__graft_entry__.smoke() and bench.py's CPU baseline): it is never part of the
product path."""
from __future__ import annotations

import json
import sys
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu)")


@lru_cache(maxsize=None)
def golden(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


def f32(bits) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint32).view(np.float32)


@lru_cache(maxsize=None)
def oracle_book(max_shell: int, min_shell: int = 2):
    from oracle.oracle import OracleBook

    return OracleBook(max_shell, min_shell)


@pytest.fixture(scope="session")
def reference_cases():
    return golden("reference_quantize.json")["cases"]


@pytest.fixture(scope="session")
def reference_tables():
    return golden("reference_tables.json")
