"""Shared pytest configuration.

`-m gpu` tests are the parity tests proper: they call the CUDA path through
the C ABI and compare with the CPU oracle.  They fail (not skip) when no CUDA
device is present, so a GPU run can never pass on a silent fallback.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; calls the CUDA path")


def pytest_runtest_setup(item):
    if item.get_closest_marker("gpu") is not None:
        import torch

        if not torch.cuda.is_available():
            pytest.fail("gpu-marked test selected but no CUDA device is available")


@pytest.fixture(scope="session")
def built_lib():
    from voom_b200 import build

    build.build()
    from voom_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def rans_cases():
    return json.loads((GOLDEN / "rans_cases.json").read_text())


@pytest.fixture(scope="session")
def rans_mutations():
    return json.loads((GOLDEN / "rans_mutations.json").read_text())


def golden_bytes(name: str) -> bytes:
    return (GOLDEN / name).read_bytes()
