"""Shared test configuration.

``-m gpu`` tests need a CUDA device (a B200); ``-m "not gpu"`` tests run on
any CPU.  Tests import the oracle from ``oracle/`` only to check results.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a library)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def digest(t: torch.Tensor | None) -> str | None:
    """SHA-256 of a tensor's bytes (BF16 viewed as int16), as in the fixtures."""
    if t is None:
        return None
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


_GOLDEN_CACHE: dict[str, dict] = {}


def golden(name: str) -> dict:
    if name not in _GOLDEN_CACHE:
        _GOLDEN_CACHE[name] = json.loads((GOLDEN / name).read_text())
    return _GOLDEN_CACHE[name]


@pytest.fixture(scope="session")
def golden_outputs() -> dict:
    return golden("golden_outputs.json")["cases"]


@pytest.fixture(scope="session")
def tile_tables() -> dict:
    return golden("tile_tables.json")["cases"]
