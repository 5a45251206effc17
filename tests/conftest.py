"""Shared fixtures. Tests marked `gpu` need a B200 (sm_100a); the rest run on CPU."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
PREBUILT = REPO / "ppy_b200" / "prebuilt"
# A checkout of the PPy reference (its `src/` holds `ppy_compiler`): the directory the
# PPY_REFERENCE environment variable names, else a checkout called `reference` beside this
# repository. Tests that run PPy's own compiler skip without one; no GPU test needs it.
REFERENCE = Path(os.environ.get("PPY_REFERENCE", str(REPO.parent / "reference")))

if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "reference: needs the PPy reference sources")


def reference_available() -> bool:
    return (REFERENCE / "src" / "ppy_compiler").exists()


@pytest.fixture(scope="session")
def ppy_compiler():
    """PPy's compiler, importable from the reference sources (CPU tests only)."""
    if not reference_available():
        pytest.skip("the PPy reference sources are not here")
    src = str(REFERENCE / "src")
    if src not in sys.path:
        sys.path.insert(0, src)
    import ppy_compiler

    return ppy_compiler


def within(actual, expected, rel: float = 1e-5, floor: float = 1.0):
    """|actual - expected| <= rel * max(|expected|, floor), NaN where expected is NaN,
    equal infinities: the 1e-5 relative fp32 tolerance, written with a floor so that it
    stays meaningful where the reference is near zero."""
    import numpy as np

    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    nan = np.isnan(expected)
    assert np.array_equal(np.isnan(actual), nan), "NaN positions differ"
    inf = np.isinf(expected)
    assert np.array_equal(actual[inf], expected[inf]), "infinities differ"
    finite = ~(nan | inf)
    scale = np.maximum(np.abs(expected[finite]), floor)
    error = np.abs(actual[finite] - expected[finite]) / scale
    worst = float(error.max()) if error.size else 0.0
    assert worst <= rel, f"max scaled error {worst:.3e} > {rel:.1e}"
    return worst
