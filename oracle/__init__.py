"""ORACLE -- test infrastructure only.

The checker the parity tests, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg
compare the B200 path against. Nothing under `ppy_b200/` imports it. It is a
restatement of the reference's CPU semantics for the hot path (`ref_loops.c`, with
the file:line of each rule it follows), compiled by `oracle/Makefile`, pinned against
the reference's own outputs in tests/golden/ (tests/test_oracle_golden.py).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_build" / "liboracle.so"

_lock = threading.Lock()
_lib = None

STATUS_OK = 0
STATUS_FALLBACK = 1


def build() -> Path:
    """Compile ref_loops.c (gcc, OpenMP) into oracle/_build/liboracle.so."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIBRARY


def _library():
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists() or LIBRARY.stat().st_mtime < (HERE / "ref_loops.c").stat().st_mtime:
                build()
            lib = ctypes.CDLL(str(LIBRARY))
            f32p = ctypes.POINTER(ctypes.c_float)
            i64 = ctypes.c_int64
            lib.oracle_gelu_chain.argtypes = [f32p, f32p, f32p, f32p, i64]
            lib.oracle_gelu_chain_omp.argtypes = [f32p, f32p, f32p, f32p, i64, ctypes.c_int]
            lib.oracle_softmax_layernorm.argtypes = [f32p, f32p, f32p, f32p, i64, i64, f32p]
            lib.oracle_softmax_layernorm_omp.argtypes = [f32p, f32p, f32p, f32p, i64, i64, f32p,
                                                         ctypes.c_int]
            lib.oracle_matmul_bias.argtypes = [f32p, f32p, f32p, f32p, i64, i64, i64]
            lib.oracle_collatz.argtypes = [i64, i64, ctypes.POINTER(i64), ctypes.POINTER(i64),
                                           ctypes.c_int]
            lib.oracle_collatz.restype = ctypes.c_int
            lib.oracle_collatz_steps.argtypes = [i64, i64, ctypes.POINTER(i64)]
            lib.oracle_collatz_steps.restype = ctypes.c_int
            _lib = lib
        return _lib


def _f32(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def threads_available() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1


def gelu_chain(a, b, c, threads: int | None = None) -> np.ndarray:
    out = np.empty_like(a)
    if threads is None:
        _library().oracle_gelu_chain(_f32(a), _f32(b), _f32(c), _f32(out), a.size)
    else:
        _library().oracle_gelu_chain_omp(_f32(a), _f32(b), _f32(c), _f32(out), a.size, threads)
    return out


def softmax_layernorm(x, gamma, beta, threads: int | None = None) -> np.ndarray:
    rows, cols = x.shape
    out = np.empty_like(x)
    if threads is None:
        work = np.empty(2 * cols, np.float32)
        _library().oracle_softmax_layernorm(_f32(x), _f32(gamma), _f32(beta), _f32(out), rows,
                                            cols, _f32(work))
    else:
        work = np.empty(2 * cols * max(threads, 1), np.float32)
        _library().oracle_softmax_layernorm_omp(_f32(x), _f32(gamma), _f32(beta), _f32(out), rows,
                                                cols, _f32(work), threads)
    return out


def matmul_bias(a, b, bias) -> np.ndarray:
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), np.float32)
    _library().oracle_matmul_bias(_f32(a), _f32(b), _f32(bias) if bias is not None else None,
                                  _f32(out), m, n, k)
    return out


def collatz(lo: int, hi: int, threads: int = 1) -> tuple[int, int, int]:
    """(status, sum of steps, max of steps) over [lo, hi)."""
    total, best = ctypes.c_int64(0), ctypes.c_int64(0)
    status = _library().oracle_collatz(lo, hi, ctypes.byref(total), ctypes.byref(best), threads)
    return status, total.value, best.value


def collatz_steps(lo: int, hi: int) -> tuple[int, np.ndarray]:
    out = np.zeros(max(hi - lo, 0), np.int64)
    status = _library().oracle_collatz_steps(
        lo, hi, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)))
    return status, out


# -- NumPy restatements for the small f64/f32 fixtures ----------------------------------------


def ext_max(a, c):
    """tensor.scalar_extremum max (ir/dialects/tensor.py:684-701): a NaN operand wins."""
    chosen = np.where(a >= c, a, c)
    return np.where(a == a, chosen, a)


def ext_min(a, c):
    chosen = np.where(a <= c, a, c)
    return np.where(a == a, chosen, a)


def fold(values: np.ndarray, kind: str, axis: int, dtype) -> np.ndarray:
    """The reference's row-major fold from the identity (lower_tensor.py:733-754)."""
    values = np.moveaxis(np.asarray(values, dtype), axis, 0)
    if kind == "add":
        acc = np.zeros(values.shape[1:], dtype)
    elif kind == "mul":
        acc = np.ones(values.shape[1:], dtype)
    elif kind == "max":
        acc = np.full(values.shape[1:], -np.inf, dtype)
    else:
        acc = np.full(values.shape[1:], np.inf, dtype)
    for item in values:
        if kind == "add":
            acc = (acc + item).astype(dtype)
        elif kind == "mul":
            acc = (acc * item).astype(dtype)
        elif kind == "max":
            acc = ext_max(acc, item)
        else:
            acc = ext_min(acc, item)
    return acc


# -- views and copies (lower_tensor.py:695-754) -----------------------------------------------


def strided(buffer: np.ndarray, shape: tuple, offset: int, strides: tuple) -> np.ndarray:
    """The reference's `_View` (lower_tensor.py:695-714): element (i0, i1, ...) of the view is
    buffer[offset + i0 * strides[0] + i1 * strides[1] + ...] of the flat `buffer`."""
    flat = np.ascontiguousarray(buffer).ravel()
    index = np.full(shape, offset, np.int64)
    for axis, (extent, stride) in enumerate(zip(shape, strides)):
        step = np.arange(extent, dtype=np.int64) * stride
        index += step.reshape((1,) * axis + (extent,) + (1,) * (len(shape) - axis - 1))
    return flat[index]


def _row_major(shape: tuple) -> tuple:
    strides, running = [1] * len(shape), 1
    for axis in reversed(range(len(shape))):
        strides[axis] = running
        running *= shape[axis]
    return tuple(strides)


def transpose(x: np.ndarray, perm: tuple) -> np.ndarray:
    """`op_transpose` (lower_tensor.py:695-702): the same memory, strides permuted."""
    strides = _row_major(x.shape)
    return strided(x, tuple(x.shape[p] for p in perm), 0, tuple(strides[p] for p in perm))


def slice_(x: np.ndarray, starts: tuple, stops: tuple, steps: tuple) -> np.ndarray:
    """`op_slice` (lower_tensor.py:704-714): offset += start * stride, stride *= step, and
    ceil((stop - start) / step) elements per axis (ir/shape.py:247-261)."""
    strides = _row_major(x.shape)
    offset = sum(start * stride for start, stride in zip(starts, strides))
    shape = tuple(-(-(stop - start) // step) for start, stop, step in zip(starts, stops, steps))
    return strided(x, shape, offset, tuple(s * k for s, k in zip(strides, steps)))


def concat(parts: list, axis: int) -> np.ndarray:
    """`op_concat` (lower_tensor.py:716-730): each part copied in at its position along axis."""
    shape = list(parts[0].shape)
    shape[axis] = sum(p.shape[axis] for p in parts)
    out = np.empty(shape, parts[0].dtype)
    position = 0
    for part in parts:
        index = [slice(None)] * len(shape)
        index[axis] = slice(position, position + part.shape[axis])
        out[tuple(index)] = part
        position += part.shape[axis]
    return out


def fold_axes(values: np.ndarray, kind: str, axes: tuple, keepdims: bool, dtype) -> np.ndarray:
    """`op_reduce` over any axes (lower_tensor.py:733-754): every output element folds its
    elements from the identity in the row-major order of the reduced axes."""
    values = np.asarray(values, dtype)
    kept = [d for d in range(values.ndim) if d not in axes]
    moved = np.transpose(values, tuple(sorted(axes)) + tuple(kept))
    flat = moved.reshape((-1,) + tuple(values.shape[d] for d in kept))
    out = fold(flat, kind, 0, dtype)
    if keepdims:
        out = out.reshape(tuple(1 if d in axes else values.shape[d] for d in range(values.ndim)))
    return out


# -- parallel bodies that call the math externs (tests/golden/parallel_math.*) ---------------


def math_table(lo: int, hi: int) -> np.ndarray:
    """out[i - lo] = tanh(x) + erf(x) + atan2(x, 1.5), x = (i - 500) * 0.01, in CPython: the
    plain run of the fixture's `math_table`. The reference's native path calls the same libm
    functions through ppy_math_unary/binary (src/ppy_runtime/stdlib.c:497-528), left to
    right, so the two agree bit for bit on one machine."""
    import math

    out = np.empty(max(hi - lo, 0), np.float64)
    for i in range(lo, hi):
        x = (i - 500) * 0.01
        out[i - lo] = math.tanh(x) + math.erf(x) + math.atan2(x, 1.5)
    return out


def asin_table(lo: int, hi: int) -> tuple[int, np.ndarray]:
    """(status, out) for the fixture's `asin_table`: out[i - lo] = asin(i * 0.25). A value
    outside [-1, 1] makes CPython raise ValueError; the native path's domain guard around
    ppy_math_unary (lowering/stdlib.py:693-731) returns STATUS_FALLBACK so that CPython reruns
    the call and raises. Status 0 with the values otherwise."""
    import math

    out = np.empty(max(hi - lo, 0), np.float64)
    for i in range(lo, hi):
        x = i * 0.25
        if not -1.0 <= x <= 1.0:
            return STATUS_FALLBACK, out
        out[i - lo] = math.asin(x)
    return STATUS_OK, out
