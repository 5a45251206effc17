"""Views and copies on the GPU, through the built module's C ABI (ppy_b200/prebuilt/views):
transposes and slices read in place by a map (strided reads of the loaded memory, the
reference's `_View`, lower_tensor.py:695-714), concat as one copy per part (:716-730),
reductions over middle axes as a transposed copy and a row reduction, and views read by a row
reduction and by a matmul through a contiguous copy, and `linalg.dot`. Against the reference's JIT outputs
(tests/golden/views.npz): bit-exact for copies, extremum and exact arithmetic; the fp32
tolerance (`within`) for exp, sums and the matmul."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, PREBUILT, within

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def views():
    from ppy_b200 import runtime

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    runtime.init(0)
    runtime.set_stream(torch.cuda.current_stream())
    return runtime.load(PREBUILT / "views" / "views.json")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "views.npz")


def _run(module, golden, name, count):
    inputs = [golden[f"{name}_in{i}"] for i in range(count)]
    out = np.full(golden[f"{name}_out"].shape, 7.0, np.float32)
    result = getattr(module, name)(*[x.ravel() for x in inputs], out.ravel())
    assert result.status == 0
    return out, golden[f"{name}_out"]


@pytest.mark.parametrize("name,count", [("transpose_add", 2), ("permute3", 1),
                                        ("concat_cols", 2), ("concat_rows", 2),
                                        ("max_split", 1)])
def test_exact_views_match_the_reference(views, golden, name, count):
    got, want = _run(views, golden, name, count)
    assert np.array_equal(got, want, equal_nan=True)


@pytest.mark.parametrize("name,count", [("slice_exp", 1), ("sum_mid", 1), ("rowsum_t", 1),
                                        ("matmul_t", 2), ("dot", 2)])
def test_rounded_views_match_the_reference(views, golden, name, count):
    got, want = _run(views, golden, name, count)
    within(got, want)


def test_a_slice_past_the_rows_falls_back(views):
    """slice_exp takes rows 2..12 of x [N, 40]: with N = 11 the call returns FALLBACK (the
    caller reruns it in CPython) and writes nothing."""
    x = np.ones((11, 40), np.float32)
    out = np.full((10, 16), 7.0, np.float32)
    assert views.slice_exp(x.ravel(), out.ravel()).status == 1
    assert np.all(out == 7.0)


def test_views_at_larger_sizes_against_the_oracle(views):
    rng = np.random.default_rng(21)
    n = 100_003
    a = rng.standard_normal((n, 32)).astype(np.float32)
    b = rng.standard_normal((32, n)).astype(np.float32)
    out = np.empty((n, 32), np.float32)
    assert views.transpose_add(a.ravel(), b.ravel(), out.ravel()).status == 0
    assert np.array_equal(out, a + np.float32(2) * oracle.transpose(b, (1, 0)))
    x = rng.standard_normal((5000, 6, 5, 7)).astype(np.float32)
    x[17, 2, 3, 6] = np.nan
    got = np.empty((5000, 1, 5, 1), np.float32)
    assert views.max_split(x.ravel(), got.ravel()).status == 0
    assert np.array_equal(got, oracle.fold_axes(x, "max", (1, 3), True, np.float32),
                          equal_nan=True)
    y = rng.standard_normal((20000, 24, 16)).astype(np.float32)
    s = np.empty((20000, 16), np.float32)
    assert views.sum_mid(y.ravel(), s.ravel()).status == 0
    within(s, oracle.fold_axes(y, "add", (1,), False, np.float64))
