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
