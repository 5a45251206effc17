"""The oracle against the reference's own outputs (tests/golden/, made by running PPy's
LLVM JIT and `ppy run` with tests/golden/make_golden.py). This pins the checker every
GPU parity test uses."""

from __future__ import annotations

import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN


@pytest.mark.parametrize("case", ["n0", "n1", "n3", "n4", "n5", "n8", "n31", "n4099", "edge"])
def test_gelu_oracle_is_bit_exact_with_the_reference(case):
    d = np.load(GOLDEN / "gelu.npz")
    out = oracle.gelu_chain(d[f"{case}_a"], d[f"{case}_b"], d[f"{case}_c"])
    assert int(d[f"{case}_status"]) == 0
    assert np.array_equal(out, d[f"{case}_out"], equal_nan=True)


def test_gelu_threads_agree_with_serial():
    rng = np.random.default_rng(3)
    a, b, c = (rng.uniform(-4, 4, 100_003).astype(np.float32) for _ in range(3))
    assert np.array_equal(oracle.gelu_chain(a, b, c), oracle.gelu_chain(a, b, c, threads=4))


def test_softmax_layernorm_oracle_is_bit_exact_with_the_reference():
    d = np.load(GOLDEN / "rows.npz")
    out = oracle.softmax_layernorm(d["x"], d["gamma"], d["beta"])
    assert int(d["status"]) == 0
    assert np.array_equal(out, d["out"])
    assert np.array_equal(oracle.softmax_layernorm(d["x"], d["gamma"], d["beta"], threads=3), out)
    # the reference's guards: an empty tensor is fine, a ragged buffer falls back
    assert int(d["empty_status"]) == 0 and int(d["ragged_status"]) == 1


def test_matmul_oracle_is_bit_exact_with_the_reference():
    d = np.load(GOLDEN / "matmul.npz")
    assert np.array_equal(oracle.matmul_bias(d["a"], d["b"], d["bias"]), d["out"])


def test_collatz_oracle_matches_ppy_run():
    g = json.loads((GOLDEN / "collatz.json").read_text())
    assert oracle.collatz(1, 1 << 16, 4)[:2] == (0, g["sum_1_65536"])
    assert oracle.collatz(1, 1000, 1)[:2] == (0, g["sum_1_1000"])
    assert oracle.collatz(27, 28, 1)[:2] == (0, g["sum_27_28"])
    assert oracle.collatz(5, 5, 1)[:2] == (0, g["sum_5_5"])
    assert oracle.collatz(1, 4096, 2)[2] == g["max_1_4096"] == g["jit_max_1_4096"][1]
    assert oracle.collatz(1, 1 << 16, 2)[2] == g["jit_max_1_65536"][1]
    status, steps = oracle.collatz_steps(1, 4096)
    assert status == 0 and steps.size == g["steps_count_1_4096"]
    assert steps[26] == g["steps_of_27"] and steps.max() == g["max_1_4096"]
    assert oracle.collatz(*g["overflow_range"], 1)[0] == g["jit_overflow_status"] == 1


def test_chain_fixtures_against_numpy_semantics():
    """The reference's own fixture values (tests/test_tensor_fusion.py:285-297)."""
    d = np.load(GOLDEN / "chain.npz")
    assert list(d["status"]) == [0, 0, 0]
    a, c = d["a"], d["c"]
    assert np.allclose(d["blend"], oracle.ext_max(np.sqrt(a) * c + 0.25, -c), rtol=0, atol=0)
    assert np.array_equal(d["energy"], (d["pairs"].reshape(4, 2) ** 2).sum(axis=1))
    assert np.array_equal(d["plus"], np.sqrt(a) + a)
    assert np.array_equal(d["minus"], np.sqrt(a) - a)


def test_reduction_fixtures_follow_the_row_major_fold():
    d = np.load(GOLDEN / "reductions.npz")
    assert list(d["status"]) == [0, 0, 0, 0]
    a = d["a"]
    assert np.array_equal(d["sumsq"], oracle.fold(a * a, "add", 0, np.float32).reshape(1))
    colmax = oracle.fold(np.abs(d["x"]), "max", 0, np.float32)
    assert np.array_equal(d["colmax"], colmax, equal_nan=True)
    assert np.isnan(d["colmax"][5])
    rowmin = oracle.fold(d["y"] - d["bias"], "min", 1, np.float32)
    assert np.array_equal(d["rowmin"], rowmin)
    prod = oracle.fold((1 + d["p"] * np.float32(0.125)).astype(np.float32).ravel(), "mul", 0,
                       np.float32)
    assert np.array_equal(d["prod"], prod.reshape(1))


def test_view_fixtures_follow_the_strided_views():
    """views.npz, from the reference's LLVM JIT: transposes and slices are strided reads of the
    loaded memory, concat copies, reductions over middle axes fold in row-major order."""
    d = np.load(GOLDEN / "views.npz")
    assert list(d["status"]) == [0] * 10
    f32 = np.float32
    a, b = d["transpose_add_in0"], d["transpose_add_in1"]
    assert np.array_equal(d["transpose_add_out"], a + f32(2) * oracle.transpose(b, (1, 0)))
    assert np.array_equal(d["permute3_out"], oracle.transpose(d["permute3_in0"], (2, 0, 1)))
    x = d["slice_exp_in0"]
    grown = np.exp(oracle.slice_(x, (2, 3), (12, 35), (1, 2)))
    want = grown - oracle.slice_(x, (0, 0), (10, 16), (1, 1))
    # NumPy's and the reference's f32 exp may differ in the last bit: bound it by the exp term
    assert np.all(np.abs(d["slice_exp_out"] - want) <= 1e-6 * np.maximum(grown, 1))
    assert np.array_equal(d["concat_cols_out"], oracle.concat(
        [d["concat_cols_in0"] * f32(2), d["concat_cols_in1"] + f32(1)], 1))
    assert np.array_equal(d["concat_rows_out"], oracle.concat(
        [d["concat_rows_in0"], np.sqrt(np.abs(d["concat_rows_in1"]))], 0))
    assert np.array_equal(d["sum_mid_out"],
                          oracle.fold_axes(d["sum_mid_in0"], "add", (1,), False, f32))
    assert np.array_equal(d["max_split_out"],
                          oracle.fold_axes(d["max_split_in0"], "max", (1, 3), True, f32),
                          equal_nan=True)
    assert np.isnan(d["max_split_out"]).sum() == 1
    assert np.array_equal(d["rowsum_t_out"], oracle.fold_axes(
        oracle.transpose(d["rowsum_t_in0"], (1, 0)), "add", (1,), False, f32))
    # linalg.dot: the products folded from zero in index order (lower_tensor.py:792-802)
    assert np.array_equal(d["dot_out"], oracle.fold(d["dot_in0"] * d["dot_in1"], "add", 0,
                                                    f32).reshape(1))
    at = oracle.transpose(d["matmul_t_in0"], (1, 0))
    assert np.allclose(d["matmul_t_out"], at.astype(np.float64) @ d["matmul_t_in1"], rtol=1e-5,
                       atol=1e-5)


def test_parallel_math_oracle_is_bit_exact_with_the_reference():
    """parallel.map and math-extern bodies (tests/golden/parallel_math.*, the reference's JIT
    with its C runtime): Collatz steps stored by the map, tanh + erf + atan2 through
    ppy_math_unary/binary, asin in its domain, and the domain guard's fallback."""
    d = np.load(GOLDEN / "parallel_math.npz")
    assert int(d["map_status"]) == 0 and int(d["map_value"]) == 4999
    status, steps = oracle.collatz_steps(1, 5000)
    assert status == 0 and np.array_equal(d["steps"][1:], steps) and d["steps"][0] == -1
    assert int(d["table_status"]) == 0 and int(d["table_value"]) == 1000
    assert np.array_equal(oracle.math_table(0, 1000), d["table"])
    status, values = oracle.asin_table(0, 5)
    assert status == int(d["asin_status"]) == 0 and np.array_equal(values, d["asin"])
    assert oracle.asin_table(0, 8)[0] == int(d["asin_bad_status"]) == oracle.STATUS_FALLBACK
