"""Locates a checkout of the reference (KyleBoyer/vOOM) for tests that run its
own, unmodified host code against this library: $VOOM_REFERENCE, else a
`reference` directory beside this repository.  The checkout is read only and
never travels with the repository, so these tests skip where it is absent
(on GPU hosts, for instance); everything they need from it is imported at
run time, nothing is copied."""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import pytest


def reference_root() -> Path | None:
    env = os.environ.get("VOOM_REFERENCE")
    cands = [Path(env)] if env else []
    cands.append(Path(__file__).resolve().parents[2] / "reference")
    for c in cands:
        if (c / "runtime" / "weight_cache.py").is_file() and (c / "formats" / "bf16_rans.py").is_file():
            return c
    return None


def reference_module(name: str):
    """Imports `name` (e.g. "runtime.weight_cache") from the reference checkout,
    or skips the calling test when there is none."""
    root = reference_root()
    if root is None:
        pytest.skip("no reference checkout (set VOOM_REFERENCE)")
    if str(root) not in sys.path:
        sys.path.append(str(root))
    mod = importlib.import_module(name)
    assert Path(mod.__file__).resolve().is_relative_to(root.resolve()), mod.__file__
    return mod
