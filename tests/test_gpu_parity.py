"""Parity of the B200 path with the reference, through the C ABI.

Every call goes through a built module's exported entry points (`<symbol>` with host
buffers, `<symbol>__device` with device buffers), on the reference's own inputs
(tests/golden/*.npz, outputs of PPy's LLVM JIT) and at BASELINE sizes against the
oracle. Tolerances: bit-exact for integer and index work; |y - ref| <= 1e-5 *
max(|ref|, 1) for fp32 (`within`).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, PREBUILT, within

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def rt():
    from ppy_b200 import runtime

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    runtime.init(0)
    # torch's current stream: the tests' copies and the module's kernels stay in order
    runtime.set_stream(torch.cuda.current_stream())
    return runtime


def _load(rt, name):
    return rt.load(PREBUILT / name / f"{name}.json")


# ---------------------------------------------------------------- fused map (config 1)


@pytest.mark.parametrize("case", ["n0", "n1", "n3", "n4", "n5", "n8", "n31", "n4099", "edge"])
def test_gelu_matches_the_reference_outputs(rt, case):
    module = _load(rt, "gelu")
    d = np.load(GOLDEN / "gelu.npz")
    a, b, c = d[f"{case}_a"], d[f"{case}_b"], d[f"{case}_c"]
    out = np.full_like(a, 7.0)
    status, value = module.gelu_chain(a, b, c, out)
    assert (status, value) == (int(d[f"{case}_status"]), 0)
    within(out, d[f"{case}_out"])


def test_gelu_full_size_against_the_oracle(rt):
    module = _load(rt, "gelu")
    rng = np.random.default_rng(0)
    n = 1 << 24
    a, b, c = (rng.uniform(-4, 4, n).astype(np.float32) for _ in range(3))
    out = np.empty_like(a)
    assert module.gelu_chain(a, b, c, out).status == 0
    expected = oracle.gelu_chain(a, b, c, threads=oracle.threads_available())
    within(out, expected)
    # the device entry point on resident tensors gives the same bits
    ta, tb, tc = (torch.from_numpy(x).cuda() for x in (a, b, c))
    tout = torch.empty_like(ta)
    assert module.device.gelu_chain(ta, tb, tc, tout).status == 0
    torch.cuda.synchronize()
    assert np.array_equal(tout.cpu().numpy(), out)


def test_gelu_from_ppy_source_matches_the_ir_module(rt):
    """tests/golden/gelu_source.ppy (PPy source over ppy.Tensor, typed by the b200_tensor
    plugin) builds the same kernel as the .ppyir fixture: the same bits, host and device."""
    module = _load(rt, "gelu_source")
    ir_module = _load(rt, "gelu")
    rng = np.random.default_rng(3)
    n = 1 << 20  # the shape the source declares
    a, b, c = (rng.uniform(-4, 4, n).astype(np.float32) for _ in range(3))
    out = np.empty_like(a)
    assert module.gelu_source_gelu_chain(a, b, c, out).status == 0
    within(out, oracle.gelu_chain(a, b, c))
    same = np.empty_like(a)
    assert ir_module.gelu_chain(a, b, c, same).status == 0
    assert np.array_equal(out, same)
    ta, tb, tc = (torch.from_numpy(x).cuda() for x in (a, b, c))
    tout = torch.empty_like(ta)
    assert module.device.gelu_source_gelu_chain(ta, tb, tc, tout).status == 0
    torch.cuda.synchronize()
    assert np.array_equal(tout.cpu().numpy(), out)
    # a buffer of another length than the declared shape takes the fallback
    short = np.empty(n - 1, np.float32)
    assert module.gelu_source_gelu_chain(a[:-1], b[:-1], c[:-1], short).status == 1


def test_gelu_unaligned_and_ragged_device_buffers(rt):
    module = _load(rt, "gelu")
    rng = np.random.default_rng(5)
    n = 10_001
    base = [torch.from_numpy(rng.uniform(-4, 4, n + 1).astype(np.float32)).cuda() for _ in range(3)]
    views = [t[1:] for t in base]  # 4-byte offset: the scalar kernel takes it
    out = torch.empty(n + 1, dtype=torch.float32, device="cuda")[1:]
    assert module.device.gelu_chain(*views, out).status == 0
    torch.cuda.synchronize()
    expected = oracle.gelu_chain(*(v.cpu().numpy().copy() for v in views))
    within(out.cpu().numpy(), expected)


def test_gelu_short_buffer_takes_the_fallback(rt):
    module = _load(rt, "gelu")
    a = np.ones(8, np.float32)
    short = np.ones(7, np.float32)
    out = np.zeros(8, np.float32)
    # N is bound from a's length; b holds fewer elements: the bounds guard fails
    assert module.gelu_chain(a, short, a, out).status == 1
    assert not out.any()


# ---------------------------------------------------------------- row group (config 3)


def test_softmax_layernorm_matches_the_reference_outputs(rt):
    module = _load(rt, "rows")
    d = np.load(GOLDEN / "rows.npz")
    out = np.zeros_like(d["x"])
    status, _ = module.softmax_layernorm(d["x"].ravel(), d["gamma"], d["beta"], out.ravel())
    assert status == int(d["status"]) == 0
    within(out, d["out"])


def test_softmax_layernorm_guards(rt):
    module = _load(rt, "rows")
    d = np.load(GOLDEN / "rows.npz")
    empty = np.zeros(0, np.float32)
    assert module.softmax_layernorm(empty, d["gamma"], d["beta"], empty).status == int(
        d["empty_status"])
    ragged = np.zeros(1024 * 2 + 7, np.float32)
    assert module.softmax_layernorm(ragged, d["gamma"], d["beta"], np.zeros_like(ragged)).status \
        == int(d["ragged_status"]) == 1


def test_softmax_layernorm_full_size_against_the_oracle(rt):
    module = _load(rt, "rows")
    rng = np.random.default_rng(0)
    x = rng.standard_normal((65536, 1024), dtype=np.float32)
    gamma = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    tx = torch.from_numpy(x).cuda()
    tg, tb = torch.from_numpy(gamma).cuda(), torch.from_numpy(beta).cuda()
    tout = torch.empty_like(tx)
    assert module.device.softmax_layernorm(tx, tg, tb, tout).status == 0
    torch.cuda.synchronize()
    expected = oracle.softmax_layernorm(x, gamma, beta, threads=oracle.threads_available())
    within(tout.cpu().numpy(), expected)
    # size-independent properties: every output row has mean(y - beta)/gamma ~ 0
    y = (tout.cpu().double().numpy() - beta) / gamma
    assert np.abs(y.mean(axis=1)).max() < 1e-4


def test_softmax_layernorm_host_call_in_row_slices(rt):
    """The host-memory call over 10 037 rows goes in slices of 2048 rows over two streams
    (the last one ragged), gamma and beta copied whole first: the same bits as the device call
    on the whole batch."""
    module = _load(rt, "rows")
    rng = np.random.default_rng(7)
    x = rng.standard_normal((10_037, 1024), dtype=np.float32)
    gamma = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    out = np.zeros_like(x)
    assert module.softmax_layernorm(x.ravel(), gamma, beta, out.ravel()).status == 0
    tout = torch.empty(x.shape, device="cuda")
    assert module.device.softmax_layernorm(torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda(),
                                           torch.from_numpy(beta).cuda(), tout).status == 0
    torch.cuda.synchronize()
    assert np.array_equal(out, tout.cpu().numpy())


# ---------------------------------------------------------------- small fixtures


def test_chain_fixtures_bit_exact(rt):
    """f64 maps and a 2-wide row sum: correctly rounded ops give the reference's bits."""
    module = _load(rt, "chain")
    d = np.load(GOLDEN / "chain.npz")
    out = np.zeros(10)
    assert module.blend(d["a"], d["c"], 0.25, out).status == 0
    assert np.array_equal(out, d["blend"])
    sums = np.zeros(4)
    assert module.energy(d["pairs"], sums).status == 0
    assert np.array_equal(sums, d["energy"])
    plus, minus = np.zeros(10), np.zeros(10)
    assert module.shared(d["a"], plus, minus).status == 0
    assert np.array_equal(plus, d["plus"]) and np.array_equal(minus, d["minus"])


def test_reduction_fixtures(rt):
    module = _load(rt, "reductions")
    d = np.load(GOLDEN / "reductions.npz")
    total = np.zeros(1, np.float32)
    assert module.sumsq(d["a"], total).status == 0
    within(total, d["sumsq"])
    colmax = np.zeros(64, np.float32)
    assert module.colmax(d["x"].ravel(), colmax).status == 0
    assert np.array_equal(colmax, d["colmax"], equal_nan=True)  # max is exact, NaN wins
    rowmin = np.zeros(77, np.float32)
    assert module.rowmin(d["y"].ravel(), d["bias"], rowmin).status == 0
    assert np.array_equal(rowmin, d["rowmin"])
    prod = np.zeros(1, np.float32)
    assert module.prod(d["p"].ravel(), prod).status == 0
    within(prod, d["prod"])


def test_whole_array_reduction_of_nothing_is_the_identity(rt):
    module = _load(rt, "reductions")
    total = np.full(1, 5.0, np.float32)
    assert module.sumsq(np.zeros(0, np.float32), total).status == 0
    assert total[0] == 0.0
    colmax = np.zeros(64, np.float32)
    assert module.colmax(np.zeros(0, np.float32), colmax).status == 0
    assert np.all(colmax == -np.inf)


def test_large_reductions_against_the_oracle(rt):
    module = _load(rt, "reductions")
    rng = np.random.default_rng(11)
    a = rng.standard_normal(1 << 22).astype(np.float32)
    total = np.zeros(1, np.float32)
    assert module.sumsq(a, total).status == 0
    within(total, [np.sum(a.astype(np.float64) ** 2)], rel=1e-5)
    x = rng.standard_normal((100_000, 64)).astype(np.float32)
    colmax = np.zeros(64, np.float32)
    assert module.colmax(x.ravel(), colmax).status == 0
    assert np.array_equal(colmax, np.abs(x).max(axis=0))
    # rows of 48: 12 four-float chunks over 8 lanes, so lanes past a row's last chunk idle;
    # at this size every staged row group and the last rows of the buffer are used
    y = rng.standard_normal((200_003, 48)).astype(np.float32)
    bias = rng.standard_normal(48).astype(np.float32)
    rowmin = np.zeros(200_003, np.float32)
    assert module.rowmin(y.ravel(), bias, rowmin).status == 0
    assert np.array_equal(rowmin, (y - bias).min(axis=1))


# ---------------------------------------------------------------- parallel.range (config 2)


def test_collatz_matches_ppy_run(rt):
    module = _load(rt, "collatz")
    g = json.loads((GOLDEN / "collatz.json").read_text())
    assert tuple(module.collatz_collatz_sum(1, 1 << 16)) == (0, g["sum_1_65536"])
    assert tuple(module.collatz_collatz_sum(1, 1000)) == tuple(g["jit_sum_1_1000"])
    assert tuple(module.collatz_collatz_sum(27, 28)) == (0, g["sum_27_28"])
    assert tuple(module.collatz_collatz_sum(5, 5)) == (0, g["sum_5_5"])
    assert tuple(module.collatz_collatz_max(1, 4096)) == tuple(g["jit_max_1_4096"])
    assert tuple(module.collatz_collatz_max(1, 1 << 16)) == tuple(g["jit_max_1_65536"])


def test_collatz_overflow_takes_the_fallback(rt):
    module = _load(rt, "collatz")
    g = json.loads((GOLDEN / "collatz.json").read_text())
    lo, hi = g["overflow_range"]
    assert module.collatz_collatz_sum(lo, hi).status == g["jit_overflow_status"] == 1
    # the status word is per call: the next call is clean
    assert tuple(module.collatz_collatz_sum(1, 1000)) == (0, g["sum_1_1000"])


def test_collatz_steps_parallel_for_writes_device_memory(rt):
    module = _load(rt, "collatz")
    g = json.loads((GOLDEN / "collatz.json").read_text())
    out = torch.zeros(4095, dtype=torch.int64, device="cuda")
    status, count = module.collatz_collatz_steps(out, 1, 4096)
    assert (status, count) == (0, g["steps_count_1_4096"])
    steps = out.cpu().numpy()
    assert steps[26] == g["steps_of_27"] and steps.max() == g["max_1_4096"]
    assert np.array_equal(steps, oracle.collatz_steps(1, 4096)[1])


def test_collatz_from_the_threads_route_matches_ppy_run(rt):
    """The same program as PPy's default `threads` route hands it over -- each range split into
    host-thread chunks (tests/golden/collatz_threads.ppyir) -- built after the backend gives
    the chunks back their range: the reference's `ppy run` answers, bit for bit."""
    module = rt.load(PREBUILT / "collatz_threads" / "collatz.json")
    g = json.loads((GOLDEN / "collatz.json").read_text())
    assert tuple(module.collatz_collatz_sum(1, 1 << 16)) == (0, g["sum_1_65536"])
    assert tuple(module.collatz_collatz_sum(27, 28)) == (0, g["sum_27_28"])
    assert tuple(module.collatz_collatz_sum(5, 5)) == (0, g["sum_5_5"])
    out = torch.zeros(4095, dtype=torch.int64, device="cuda")
    status, count = module.collatz_collatz_steps(out, 1, 4096)
    assert (status, count) == (0, g["steps_count_1_4096"])
    assert np.array_equal(out.cpu().numpy(), oracle.collatz_steps(1, 4096)[1])


def test_collatz_large_range_against_the_oracle(rt):
    module = _load(rt, "collatz")
    hi = 1 << 24
    status, total, best = oracle.collatz(1, hi, oracle.threads_available())
    assert status == 0
    assert tuple(module.collatz_collatz_sum(1, hi)) == (0, total)
    assert tuple(module.collatz_collatz_max(1, hi)) == (0, best)


def test_a_body_that_never_ends_raises_instead_of_hanging(rt):
    """Collatz from 0 never reaches 1 (the reference spins forever on the CPU); the
    device copy of the body stops at its loop bound and the call raises."""
    module = _load(rt, "collatz")
    with pytest.raises(rt.B200Error, match="trip bound"):
        module.collatz_collatz_sum(0, 1)
    g = json.loads((GOLDEN / "collatz.json").read_text())
    assert tuple(module.collatz_collatz_sum(1, 1000)) == (0, g["sum_1_1000"])


# ---------------------------------------------------------------- parallel.map and math externs


def _pmath(rt):
    return rt.load(PREBUILT / "parallel_math" / "pmath.json")


def test_parallel_map_stores_every_index_bit_exact(rt):
    """`parallel.map @collatz_steps_of() lo, hi, out` (built with the reference's map_
    builder, ir/dialects/parallel.py:184): out[i] = steps(i) for i in [1, 5000), out[0]
    untouched, exactly the reference JIT's values and the oracle's."""
    module = _pmath(rt)
    d = np.load(GOLDEN / "parallel_math.npz")
    out = torch.full((5000,), -1, dtype=torch.int64, device="cuda")
    assert tuple(module.pmath_collatz_map(out, 1, 5000)) == (int(d["map_status"]),
                                                            int(d["map_value"]))
    assert np.array_equal(out.cpu().numpy(), d["steps"])
    assert np.array_equal(out.cpu().numpy()[1:], oracle.collatz_steps(1, 5000)[1])
    # a large range against the oracle, and an empty one that writes nothing
    big = torch.zeros(1 << 20, dtype=torch.int64, device="cuda")
    assert module.pmath_collatz_map(big, 1, 1 << 20).status == 0
    assert np.array_equal(big.cpu().numpy()[1:], oracle.collatz_steps(1, 1 << 20)[1])
    assert tuple(module.pmath_collatz_map(out, 7, 7)) == (0, 0)


def test_math_externs_in_a_parallel_body(rt):
    """tanh + erf + atan2 through ppy_math_unary/binary in a parallel.for body, against the
    reference JIT's values (libm). CUDA's double tanh, erf and atan2 are within 2 ulp of the
    correctly rounded result, so the sum of three is within a few ulp:
    |y - ref| <= 1e-14 * max(|ref|, 1)."""
    module = _pmath(rt)
    d = np.load(GOLDEN / "parallel_math.npz")
    out = torch.zeros(1000, dtype=torch.float64, device="cuda")
    assert tuple(module.pmath_math_table(out, 0, 1000)) == (int(d["table_status"]),
                                                           int(d["table_value"]))
    within(out.cpu().numpy(), d["table"], rel=1e-14)
    within(out.cpu().numpy(), oracle.math_table(0, 1000), rel=1e-14)


def test_math_domain_guard_takes_the_fallback(rt):
    """asin(i / 4): in its domain for i < 5 (values within 1e-14), and for [0, 8) asin(1.25)
    fails the domain guard around the extern: FALLBACK, as the reference's JIT returns."""
    module = _pmath(rt)
    d = np.load(GOLDEN / "parallel_math.npz")
    out = torch.zeros(8, dtype=torch.float64, device="cuda")
    assert module.pmath_asin_table(out, 0, 5).status == int(d["asin_status"]) == 0
    within(out[:5].cpu().numpy(), d["asin"], rel=1e-14)
    assert module.pmath_asin_table(out, 0, 8).status == int(d["asin_bad_status"]) == 1
    # the status word is per call: the next call is clean
    assert module.pmath_asin_table(out, 0, 5).status == 0


def test_host_memory_call_in_slices_matches_the_device_call(rt):
    """An elementwise function called with host memory runs in slices of 2^21 elements over
    two streams (copies in, kernel, copies out per slice) once it has at least two slices:
    the outputs equal the device entry point's bit for bit, a ragged last slice included,
    from pinned and from pageable host memory."""
    module = _load(rt, "gelu")
    n = 5 * (1 << 21) + 123
    rng = np.random.default_rng(21)
    a, b, c = (rng.uniform(-4, 4, n).astype(np.float32) for _ in range(3))
    ta, tb, tc = (torch.from_numpy(x).cuda() for x in (a, b, c))
    want = torch.empty_like(ta)
    assert module.device.gelu_chain(ta, tb, tc, want).status == 0
    torch.cuda.synchronize()
    want = want.cpu().numpy()
    pageable = np.full(n, np.nan, np.float32)
    assert module.gelu_chain(a, b, c, pageable).status == 0
    assert np.array_equal(pageable, want)
    pa, pb, pc = (torch.from_numpy(x).pin_memory() for x in (a, b, c))
    pinned = torch.full((n,), float("nan")).pin_memory()
    assert module.gelu_chain(pa, pb, pc, pinned).status == 0
    assert np.array_equal(pinned.numpy(), want)
    within(want[: 1 << 16], oracle.gelu_chain(a[: 1 << 16], b[: 1 << 16], c[: 1 << 16]))
