"""Generate the golden fixtures under tests/golden/ by running the PPy reference.

This script is the only place the reference compiler is executed. It needs the
reference sources on PYTHONPATH (``--reference /path/to/PPy``) and llvmlite; it
writes:

* ``<name>.ppyir`` -- canonical IR after PPy's shared passes with
  ``lower_tensors=False`` (tensor modules) or the ``openmp`` parallel setting
  (parallel modules): exactly what an installed backend receives from
  ``ppy build X --backend b200`` (driver/commands.py:609-674, :677-736).
* ``<name>.npz`` -- seeded inputs and the outputs of the reference's own LLVM
  JIT of the same IR (tensor IR through ``optimize_shared_ir`` + ``LowerTensor``
  + ``JitEngine``, the road of tests/test_tensor_fusion.py:265-305), with the
  status each call returned.
* ``collatz.json`` -- ``ppy run`` output of the Collatz program (LLVM backend,
  ``threads``) and the JIT status of an overflowing range.

Run:  python tests/golden/make_golden.py --reference <a PPy checkout>  (or set PPY_REFERENCE)
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import textwrap
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _setup(reference: Path) -> None:
    sys.path.insert(0, str(reference / "src"))


# -- module builders (the reference's Builder API) ---------------------------------------


def build_gelu():
    from ppy_compiler.ir import F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    n = shapes.Symbol("N")
    buf = BufferType(F32)
    m = IRModule("gelu")
    m.require("tensor", 1)
    vec = tensor.tensor_type(F32, (n,))
    f = m.add_function("gelu_chain", [("a", buf), ("b", buf), ("c", buf), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    a_, b_, c_, out = f.entry.arguments
    ta = tensor.load(b, a_, vec, "a")
    tb = tensor.load(b, b_, vec, "b")
    tc = tensor.load(b, c_, vec, "c")

    def k(v):
        return tensor.fill(b, core.const(b, v, F32), vec)

    ew = lambda name, x, y: tensor.elementwise(b, name, x, y)  # noqa: E731
    # z = a*b + c; gelu_tanh(z) = 0.5 z (1 + tanh(sqrt(2/pi) (z + 0.044715 z^3))),
    # tanh(u) spelled 1 - 2/(exp(2u) + 1): the tensor dialect has no tanh.
    z = ew("add", ew("mul", ta, tb), tc)
    z3 = ew("mul", z, ew("mul", z, z))
    u = ew("mul", k(0.7978845608028654), ew("add", z, ew("mul", k(0.044715), z3)))
    e = tensor.unary(b, "exp", ew("mul", k(2.0), u))
    t = ew("sub", k(1.0), ew("div", k(2.0), ew("add", e, k(1.0))))
    y = ew("mul", ew("mul", k(0.5), z), ew("add", k(1.0), t))
    tensor.store(b, y, out)
    core.ret(b, core.const(b, 0, I64))
    return m


def build_rows(cols: int = 1024):
    from ppy_compiler.ir import F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    r = shapes.Symbol("R")
    buf = BufferType(F32)
    m = IRModule("rows")
    m.require("tensor", 1)
    mat = tensor.tensor_type(F32, (r, cols))
    col = tensor.tensor_type(F32, (r, 1))
    vec = tensor.tensor_type(F32, (cols,))
    f = m.add_function(
        "softmax_layernorm", [("x", buf), ("gamma", buf), ("beta", buf), ("out", buf)], [I64]
    )
    b = Builder(f.add_entry_block())
    xb, gb, bb, out = f.entry.arguments
    x = tensor.load(b, xb, mat, "x")
    g = tensor.load(b, gb, vec, "gamma")
    be = tensor.load(b, bb, vec, "beta")
    ew = lambda name, p, q: tensor.elementwise(b, name, p, q)  # noqa: E731

    def k(v):
        return tensor.fill(b, core.const(b, v, F32), col)

    mx = tensor.reduce(b, x, (1,), "max", keepdims=True)
    e = tensor.unary(b, "exp", ew("sub", x, mx))
    s = tensor.reduce(b, e, (1,), "add", keepdims=True)
    p = ew("div", e, s)
    mu = ew("div", tensor.reduce(b, p, (1,), "add", keepdims=True), k(float(cols)))
    d = ew("sub", p, mu)
    var = ew("div", tensor.reduce(b, ew("mul", d, d), (1,), "add", keepdims=True), k(float(cols)))
    rstd = ew("div", k(1.0), tensor.unary(b, "sqrt", ew("add", var, k(1e-5))))
    y = ew("add", ew("mul", ew("mul", d, rstd), g), be)
    tensor.store(b, y, out)
    core.ret(b, core.const(b, 0, I64))
    return m


def build_layernorm(cols: int = 768):
    """GPT-2's layernorm as tensor IR: f32 rows in, bf16 rows out (the next matmul's A)."""
    from ppy_compiler.ir import BF16, F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    r = shapes.Symbol("R")
    m = IRModule("gpt2_layernorm")
    m.require("tensor", 1)
    mat = tensor.tensor_type(F32, (r, cols))
    col = tensor.tensor_type(F32, (r, 1))
    vec = tensor.tensor_type(F32, (cols,))
    f = m.add_function("layernorm_bf16", [("x", BufferType(F32)), ("gamma", BufferType(F32)),
                                          ("beta", BufferType(F32)), ("out", BufferType(BF16))],
                       [I64])
    b = Builder(f.add_entry_block())
    xb, gb, bb, out = f.entry.arguments
    x = tensor.load(b, xb, mat, "x")
    g = tensor.load(b, gb, vec, "gamma")
    be = tensor.load(b, bb, vec, "beta")
    ew = lambda name, p, q: tensor.elementwise(b, name, p, q)  # noqa: E731

    def k(v):
        return tensor.fill(b, core.const(b, v, F32), col)

    mean = ew("div", tensor.reduce(b, x, (1,), "add", keepdims=True), k(float(cols)))
    d = ew("sub", x, mean)
    var = ew("div", tensor.reduce(b, ew("mul", d, d), (1,), "add", keepdims=True), k(float(cols)))
    rstd = ew("div", k(1.0), tensor.unary(b, "sqrt", ew("add", var, k(1e-5))))
    y = ew("add", ew("mul", ew("mul", d, rstd), g), be)
    tensor.store(b, tensor.convert(b, y, BF16), out)
    core.ret(b, core.const(b, 0, I64))
    return m


def build_chain():
    """The reference's own fusion fixture (tests/test_tensor_fusion.py:133-163), f64."""
    from ppy_compiler.ir import F64, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    n = shapes.Symbol("N")
    buf = BufferType(F64)
    module = IRModule("chain")
    module.require("tensor", 1)
    vector = tensor.tensor_type(F64, (n,))
    f = module.add_function("blend", [("a", buf), ("b", buf), ("s", F64), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    a, c, s, out = (f.entry.arguments[i] for i in range(4))
    ta = tensor.load(b, a, vector, "a")
    tb = tensor.load(b, c, vector, "b")
    root = tensor.unary(b, "sqrt", ta)
    scaled = tensor.elementwise(b, "mul", root, tb)
    shifted = tensor.elementwise(b, "add", scaled, tensor.fill(b, s, vector))
    tensor.store(b, tensor.elementwise(b, "max", shifted, tensor.unary(b, "neg", tb)), out)
    core.ret(b, core.const(b, 0, I64))
    g = module.add_function("energy", [("a", buf), ("out", buf)], [I64])
    b = Builder(g.add_entry_block())
    a, out = g.entry.arguments[0], g.entry.arguments[1]
    ta = tensor.load(b, a, tensor.tensor_type(F64, (n, 2)), "a")
    squared = tensor.elementwise(b, "mul", ta, ta)
    tensor.store(b, tensor.reduce(b, squared, (1,), "add"), out)
    core.ret(b, core.const(b, 0, I64))
    h = module.add_function("shared", [("a", buf), ("out", buf), ("out2", buf)], [I64])
    b = Builder(h.add_entry_block())
    a, out, out2 = (h.entry.arguments[i] for i in range(3))
    ta = tensor.load(b, a, vector, "a")
    root = tensor.unary(b, "sqrt", ta)
    tensor.store(b, tensor.elementwise(b, "add", root, ta), out)
    tensor.store(b, tensor.elementwise(b, "sub", root, ta), out2)
    core.ret(b, core.const(b, 0, I64))
    return module


def build_reductions():
    """f32 whole-array and column reductions, NaN-propagating max, and broadcasts."""
    from ppy_compiler.ir import F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    n = shapes.Symbol("N")
    buf = BufferType(F32)
    m = IRModule("reductions")
    m.require("tensor", 1)
    # total = sum(a*a) over the whole vector
    f = m.add_function("sumsq", [("a", buf), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    a, out = f.entry.arguments
    ta = tensor.load(b, a, tensor.tensor_type(F32, (n,)))
    tensor.store(b, tensor.reduce(b, tensor.elementwise(b, "mul", ta, ta), (0,), "add"), out)
    core.ret(b, core.const(b, 0, I64))
    # colmax = max over rows of |x| (axis 0 of [N, 64])
    f = m.add_function("colmax", [("x", buf), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    x, out = f.entry.arguments
    tx = tensor.load(b, x, tensor.tensor_type(F32, (n, 64)))
    tensor.store(b, tensor.reduce(b, tensor.unary(b, "abs", tx), (0,), "max"), out)
    core.ret(b, core.const(b, 0, I64))
    # rowmin = min over each row of x - bias (axis 1 of [N, 48]); bias [48] broadcast
    f = m.add_function("rowmin", [("x", buf), ("bias", buf), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    x, bias, out = f.entry.arguments
    tx = tensor.load(b, x, tensor.tensor_type(F32, (n, 48)))
    tb = tensor.load(b, bias, tensor.tensor_type(F32, (48,)))
    tensor.store(b, tensor.reduce(b, tensor.elementwise(b, "sub", tx, tb), (1,), "min"), out)
    core.ret(b, core.const(b, 0, I64))
    # prod of (1 + x/8) over the whole [N, 3] tensor
    f = m.add_function("prod", [("x", buf), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    x, out = f.entry.arguments
    t3 = tensor.tensor_type(F32, (n, 3))
    tx = tensor.load(b, x, t3)
    one = tensor.fill(b, core.const(b, 1.0, F32), t3)
    eighth = tensor.fill(b, core.const(b, 0.125, F32), t3)
    v = tensor.elementwise(b, "add", one, tensor.elementwise(b, "mul", tx, eighth))
    tensor.store(b, tensor.reduce(b, v, (0, 1), "mul"), out)
    core.ret(b, core.const(b, 0, I64))
    return m


def build_views():
    """Views and copies (f32): transpose, slice, concat, reductions over middle axes, views
    read by a row reduction and by a matmul, and `linalg.dot`."""
    from ppy_compiler.ir import F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    n = shapes.Symbol("N")
    buf = BufferType(F32)
    T = tensor.tensor_type
    m = IRModule("views")
    m.require("tensor", 1)

    def fn(name, params):
        f = m.add_function(name, [(p, buf) for p in params], [I64])
        return f, Builder(f.add_entry_block()), f.entry.arguments

    def const(b, value, shape):
        return tensor.fill(b, core.const(b, value, F32), T(F32, shape))

    # out[N, 32] = a + 2 * b^T, b [32, N]
    f, b, (a, bb, out) = fn("transpose_add", ("a", "b", "out"))
    ta = tensor.load(b, a, T(F32, (n, 32)))
    tbt = tensor.transpose(b, tensor.load(b, bb, T(F32, (32, n))), (1, 0))
    tensor.store(b, tensor.elementwise(b, "add", ta, tensor.elementwise(
        b, "mul", const(b, 2.0, (n, 32)), tbt)), out)
    core.ret(b, core.const(b, 0, I64))
    # out[N, 4, 8] = x permuted (2, 0, 1), x [4, 8, N]
    f, b, (x, out) = fn("permute3", ("x", "out"))
    tx = tensor.load(b, x, T(F32, (4, 8, n)))
    tensor.store(b, tensor.transpose(b, tx, (2, 0, 1)), out)
    core.ret(b, core.const(b, 0, I64))
    # out[10, 16] = exp(x[2:12, 3:35:2]) - x[0:10, 0:16], x [N, 40] (N >= 12)
    f, b, (x, out) = fn("slice_exp", ("x", "out"))
    tx = tensor.load(b, x, T(F32, (n, 40)))
    odd = tensor.slice_(b, tx, (2, 3), (12, 35), (1, 2))
    head = tensor.slice_(b, tx, (0, 0), (10, 16), (1, 1))
    tensor.store(b, tensor.elementwise(b, "sub", tensor.unary(b, "exp", odd), head), out)
    core.ret(b, core.const(b, 0, I64))
    # out[N, 24] = concat(2 a, b + 1) along the columns, a [N, 16], b [N, 8]
    f, b, (a, bb, out) = fn("concat_cols", ("a", "b", "out"))
    ta = tensor.load(b, a, T(F32, (n, 16)))
    tb = tensor.load(b, bb, T(F32, (n, 8)))
    left = tensor.elementwise(b, "mul", ta, const(b, 2.0, (n, 16)))
    right = tensor.elementwise(b, "add", tb, const(b, 1.0, (n, 8)))
    tensor.store(b, tensor.concat(b, (left, right), 1), out)
    core.ret(b, core.const(b, 0, I64))
    # out[16, 16] = concat(a, sqrt(|b|)) along the rows, a [6, 16], b [10, 16]
    f, b, (a, bb, out) = fn("concat_rows", ("a", "b", "out"))
    ta = tensor.load(b, a, T(F32, (6, 16)))
    tb = tensor.load(b, bb, T(F32, (10, 16)))
    tensor.store(b, tensor.concat(b, (ta, tensor.unary(b, "sqrt", tensor.unary(b, "abs", tb))),
                                  0), out)
    core.ret(b, core.const(b, 0, I64))
    # out[N, 16] = sum over the middle axis of x [N, 24, 16]
    f, b, (x, out) = fn("sum_mid", ("x", "out"))
    tx = tensor.load(b, x, T(F32, (n, 24, 16)))
    tensor.store(b, tensor.reduce(b, tx, (1,), "add"), out)
    core.ret(b, core.const(b, 0, I64))
    # out[N, 1, 5, 1] = max over axes 1 and 3 of x [N, 6, 5, 7] (keepdims)
    f, b, (x, out) = fn("max_split", ("x", "out"))
    tx = tensor.load(b, x, T(F32, (n, 6, 5, 7)))
    tensor.store(b, tensor.reduce(b, tx, (1, 3), "max", keepdims=True), out)
    core.ret(b, core.const(b, 0, I64))
    # out[N] = row sums of x^T, x [32, N]
    f, b, (x, out) = fn("rowsum_t", ("x", "out"))
    tx = tensor.load(b, x, T(F32, (32, n)))
    tensor.store(b, tensor.reduce(b, tensor.transpose(b, tx, (1, 0)), (1,), "add"), out)
    core.ret(b, core.const(b, 0, I64))
    # out[N, 24] = a^T @ w, a [32, N], w [32, 24]
    f, b, (a, w, out) = fn("matmul_t", ("a", "w", "out"))
    ta = tensor.transpose(b, tensor.load(b, a, T(F32, (32, n))), (1, 0))
    tw = tensor.load(b, w, T(F32, (32, 24)))
    tensor.store(b, tensor.matmul(b, ta, tw), out)
    core.ret(b, core.const(b, 0, I64))
    # out[] = linalg.dot(a, b), a b [1001] (the reference lowers linalg on static shapes)
    from ppy_compiler.ir.dialects import linalg

    m.require("linalg", 1)
    f, b, (a, bb, out) = fn("dot", ("a", "b", "out"))
    ta = tensor.load(b, a, T(F32, (1001,)))
    tb = tensor.load(b, bb, T(F32, (1001,)))
    tensor.store(b, linalg.dot(b, ta, tb), out)
    core.ret(b, core.const(b, 0, I64))
    return m


def build_matmul(k: int = 96, n: int = 80):
    """C = A @ B + bias, f32, A [M, K] with M symbolic."""
    from ppy_compiler.ir import F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    msym = shapes.Symbol("M")
    buf = BufferType(F32)
    mod = IRModule("matmul")
    mod.require("tensor", 1)
    f = mod.add_function("matmul_bias", [("a", buf), ("b", buf), ("bias", buf), ("out", buf)], [I64])
    b = Builder(f.add_entry_block())
    a, bb, bias, out = f.entry.arguments
    ta = tensor.load(b, a, tensor.tensor_type(F32, (msym, k)), "a")
    tb = tensor.load(b, bb, tensor.tensor_type(F32, (k, n)), "b")
    tbias = tensor.load(b, bias, tensor.tensor_type(F32, (n,)), "bias")
    prod = tensor.matmul(b, ta, tb)
    tensor.store(b, tensor.elementwise(b, "add", prod, tbias), out)
    core.ret(b, core.const(b, 0, I64))
    return mod


def build_matmul_bf16(k: int = 128, n: int = 256):
    """C = f32(A) @ f32(B) + bias with A, B bf16: bf16 operands, f32 accumulate and result.

    The reference's LowerTensor refuses bfloat16 (lower_tensor.py:119-124), so this
    module has no reference JIT output; its golden values come from NumPy.
    """
    from ppy_compiler.ir import BF16, F32, I64, BufferType, Builder, IRModule
    from ppy_compiler.ir import shape as shapes
    from ppy_compiler.ir.dialects import core, tensor

    msym = shapes.Symbol("M")
    mod = IRModule("matmul_bf16")
    mod.require("tensor", 1)
    f = mod.add_function(
        "matmul_bias_bf16",
        [("a", BufferType(BF16)), ("b", BufferType(BF16)), ("bias", BufferType(F32)),
         ("out", BufferType(F32))],
        [I64],
    )
    b = Builder(f.add_entry_block())
    a, bb, bias, out = f.entry.arguments
    ta = tensor.load(b, a, tensor.tensor_type(BF16, (msym, k)), "a")
    tb = tensor.load(b, bb, tensor.tensor_type(BF16, (k, n)), "b")
    tbias = tensor.load(b, bias, tensor.tensor_type(F32, (n,)), "bias")
    fa = tensor.convert(b, ta, F32)
    fb = tensor.convert(b, tb, F32)
    tensor.store(b, tensor.elementwise(b, "add", tensor.matmul(b, fa, fb), tbias), out)
    core.ret(b, core.const(b, 0, I64))
    return mod


# -- running the reference ------------------------------------------------------------------


def shared_passes(module, lower_tensors: bool):
    from ppy_compiler.backend.llvm.ir_pipeline import optimize

    optimize(module, 2, lower_tensors=lower_tensors)
    return module


def jit(module):
    from ppy_compiler.backend.llvm.from_ir import emit_module
    from ppy_compiler.backend.llvm.jit import JitEngine

    engine = JitEngine(opt_level=2).open()
    engine.add(emit_module(module))
    engine.finalize()
    return engine


def call(engine, symbol, *arguments):
    """Call a JIT'd tensor function with the LLVM ABI: (ptr, len) per buffer, scalars
    by value, then the result slot; returns the status."""
    atoms, kinds = [], []
    for argument in arguments:
        if isinstance(argument, np.ndarray):
            ctype = {np.float32: ctypes.c_float, np.float64: ctypes.c_double,
                     np.int64: ctypes.c_int64}[argument.dtype.type]
            pointer = ctypes.POINTER(ctype)
            atoms.extend([argument.ctypes.data_as(pointer), argument.size])
            kinds.extend([pointer, ctypes.c_int64])
        elif isinstance(argument, float):
            atoms.append(argument)
            kinds.append(ctypes.c_double)
        else:
            atoms.append(int(argument))
            kinds.append(ctypes.c_int64)
    slot = ctypes.c_int64(0)
    fn = ctypes.CFUNCTYPE(ctypes.c_int32, *kinds, ctypes.POINTER(ctypes.c_int64))(
        engine.address(symbol)
    )
    return int(fn(*atoms, ctypes.byref(slot))), int(slot.value)


def write_ppyir(module, name: str) -> None:
    """Encode `module` as .ppyir. FuseTensor names every fused body `^body`, and the
    reference's parser refuses a second `^body` in one function ("^body is defined
    twice"), so bodies are renumbered first; nothing else changes."""
    from ppy_compiler.ir import decode, encode

    for function in module.functions.values():
        count = 0
        for op in function.operations():
            for region in op.regions:
                for block in region.blocks:
                    block.name = f"body{count}"
                    count += 1
    text = encode(module)
    decode(text)  # the backend's road reads it back
    (HERE / f"{name}.ppyir").write_text(text, encoding="utf-8")


def golden_gelu() -> None:
    write_ppyir(shared_passes(build_gelu(), False), "gelu")
    engine = jit(shared_passes(build_gelu(), True))
    rng = np.random.default_rng(0)
    cases = {}
    for n in (0, 1, 3, 4, 5, 8, 31, 4099):
        a, b, c = (rng.uniform(-4, 4, n).astype(np.float32) for _ in range(3))
        out = np.zeros(n, np.float32)
        status, _ = call(engine, "gelu_chain", a, b, c, out)
        cases[f"n{n}"] = (a, b, c, out, status)
    # Edge values: large magnitudes (exp overflows to inf), zeros, a NaN.
    edge = np.array([0.0, -0.0, 1e-30, -9.0, 9.0, 40.0, -40.0, np.nan, np.inf, -np.inf, 88.0,
                     -88.0], np.float32)
    ones = np.ones_like(edge)
    zeros = np.zeros_like(edge)
    out = np.zeros_like(edge)
    status, _ = call(engine, "gelu_chain", edge, ones, zeros, out)
    cases["edge"] = (edge, ones, zeros, out, status)
    arrays = {}
    for key, (a, b, c, out, status) in cases.items():
        arrays.update({f"{key}_a": a, f"{key}_b": b, f"{key}_c": c, f"{key}_out": out,
                       f"{key}_status": np.int32(status)})
    np.savez_compressed(HERE / "gelu.npz", **arrays)


def golden_rows() -> None:
    write_ppyir(shared_passes(build_rows(), False), "rows")
    engine = jit(shared_passes(build_rows(), True))
    rng = np.random.default_rng(0)
    rows = 37
    x = rng.standard_normal((rows, 1024), dtype=np.float32)
    x[3] *= 30.0  # a row with a wide range: exp underflows for most of it
    x[5] = 0.0  # a constant row: variance 0, the output is beta
    gamma = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    beta = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    out = np.zeros_like(x)
    status, _ = call(engine, "softmax_layernorm", x.ravel(), gamma, beta, out.ravel())
    empty = np.zeros((0, 1024), np.float32)
    empty_status, _ = call(engine, "softmax_layernorm", empty.ravel(), gamma, beta,
                           empty.ravel())
    # A buffer whose length is not a multiple of 1024 fails the binding guard.
    ragged = np.zeros(1024 * 2 + 7, np.float32)
    ragged_status, _ = call(engine, "softmax_layernorm", ragged, gamma, beta,
                            np.zeros_like(ragged))
    np.savez_compressed(HERE / "rows.npz", x=x, gamma=gamma, beta=beta, out=out,
                        status=np.int32(status), empty_status=np.int32(empty_status),
                        ragged_status=np.int32(ragged_status))


def golden_chain() -> None:
    write_ppyir(shared_passes(build_chain(), False), "chain")
    engine = jit(shared_passes(build_chain(), True))
    a = np.linspace(0.0, 9.0, 10)
    c = np.linspace(-1.0, 1.0, 10)
    out = np.zeros(10)
    s1, _ = call(engine, "blend", a, c, 0.25, out)
    pairs = np.arange(8, dtype=np.float64)
    sums = np.zeros(4)
    s2, _ = call(engine, "energy", pairs, sums)
    plus, minus = np.zeros(10), np.zeros(10)
    s3, _ = call(engine, "shared", a, plus, minus)
    np.savez_compressed(HERE / "chain.npz", a=a, c=c, blend=out, pairs=pairs, energy=sums,
                        plus=plus, minus=minus, status=np.array([s1, s2, s3], np.int32))


def golden_reductions() -> None:
    write_ppyir(shared_passes(build_reductions(), False), "reductions")
    engine = jit(shared_passes(build_reductions(), True))
    rng = np.random.default_rng(1)
    a = rng.standard_normal(10007).astype(np.float32)
    total = np.zeros(1, np.float32)
    s1, _ = call(engine, "sumsq", a, total)
    x = rng.standard_normal((129, 64)).astype(np.float32)
    x[7, 5] = np.nan
    colmax = np.zeros(64, np.float32)
    s2, _ = call(engine, "colmax", x.ravel(), colmax)
    y = rng.standard_normal((77, 48)).astype(np.float32)
    bias = rng.standard_normal(48).astype(np.float32)
    rowmin = np.zeros(77, np.float32)
    s3, _ = call(engine, "rowmin", y.ravel(), bias, rowmin)
    p = rng.uniform(-1, 1, (50, 3)).astype(np.float32)
    prod = np.zeros(1, np.float32)
    s4, _ = call(engine, "prod", p.ravel(), prod)
    np.savez_compressed(HERE / "reductions.npz", a=a, sumsq=total, x=x, colmax=colmax, y=y,
                        bias=bias, rowmin=rowmin, p=p, prod=prod,
                        status=np.array([s1, s2, s3, s4], np.int32))


def golden_views() -> None:
    write_ppyir(shared_passes(build_views(), False), "views")
    engine = jit(shared_passes(build_views(), True))
    rng = np.random.default_rng(4)
    f32 = np.float32
    arrays, status = {}, []

    def run(name, inputs, out_shape):
        out = np.zeros(out_shape, f32)
        st, _ = call(engine, name, *[x.ravel() for x in inputs], out.ravel())
        status.append(st)
        for i, x in enumerate(inputs):
            arrays[f"{name}_in{i}"] = x
        arrays[f"{name}_out"] = out

    run("transpose_add", [rng.standard_normal((37, 32)).astype(f32),
                          rng.standard_normal((32, 37)).astype(f32)], (37, 32))
    run("permute3", [rng.standard_normal((4, 8, 29)).astype(f32)], (29, 4, 8))
    run("slice_exp", [rng.standard_normal((13, 40)).astype(f32)], (10, 16))
    run("concat_cols", [rng.standard_normal((21, 16)).astype(f32),
                        rng.standard_normal((21, 8)).astype(f32)], (21, 24))
    run("concat_rows", [rng.standard_normal((6, 16)).astype(f32),
                        rng.standard_normal((10, 16)).astype(f32)], (16, 16))
    run("sum_mid", [rng.standard_normal((9, 24, 16)).astype(f32)], (9, 16))
    x = rng.standard_normal((4, 6, 5, 7)).astype(f32)
    x[2, 3, 1, 4] = np.nan
    run("max_split", [x], (4, 1, 5, 1))
    run("rowsum_t", [rng.standard_normal((32, 50)).astype(f32)], (50,))
    run("matmul_t", [rng.standard_normal((32, 40)).astype(f32),
                     rng.standard_normal((32, 24)).astype(f32)], (40, 24))
    run("dot", [rng.standard_normal(1001).astype(f32), rng.standard_normal(1001).astype(f32)],
        (1,))
    np.savez_compressed(HERE / "views.npz", status=np.array(status, np.int32), **arrays)


def golden_matmul() -> None:
    write_ppyir(shared_passes(build_matmul(), False), "matmul")
    engine = jit(shared_passes(build_matmul(), True))
    rng = np.random.default_rng(0)
    m, k, n = 64, 96, 80
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    bias = (0.02 * rng.standard_normal(n)).astype(np.float32)
    out = np.zeros((m, n), np.float32)
    status, _ = call(engine, "matmul_bias", a.ravel(), b.ravel(), bias, out.ravel())
    np.savez_compressed(HERE / "matmul.npz", a=a, b=b, bias=bias, out=out,
                        status=np.int32(status))
    # The bf16 modules: their IR only (the reference refuses to lower bf16 tensors).
    write_ppyir(shared_passes(build_matmul_bf16(), False), "matmul_bf16")
    # the benchmark shape: C = A @ B + bias with M = N = K = 8192 (M bound at run time)
    module = build_matmul_bf16(k=8192, n=8192)
    module.name = "matmul_bf16_8192"
    write_ppyir(shared_passes(module, False), "matmul_bf16_8192")
    # the fp32-input variant's benchmark shape: M = N = K = 4096 (M bound at run time); its
    # IR only (the reference's naive loop nest would take hours at this size)
    module = build_matmul(k=4096, n=4096)
    module.name = "matmul_f32_4096"
    write_ppyir(shared_passes(module, False), "matmul_f32_4096")


COLLATZ = '''
from ppy import native, parallel


def collatz_sum(lo: int, hi: int) -> int:
    total = 0
    for start in parallel.range(lo, hi):
        x = start
        steps = 0
        while x != 1:
            if x % 2 == 0:
                x = x // 2
            else:
                x = 3 * x + 1
            steps += 1
        total += steps
    return total


def collatz_steps(out: native.ptr[int], lo: int, hi: int) -> int:
    for start in parallel.range(lo, hi):
        x = start
        steps = 0
        while x != 1:
            if x % 2 == 0:
                x = x // 2
            else:
                x = 3 * x + 1
            steps += 1
        native.store(native.offset(out, start - lo), steps)
    return hi - lo
'''

COLLATZ_MAIN = '''

def main() -> None:
    print(collatz_sum(1, 1 << 16))
    print(collatz_sum(1, 1000))
    print(collatz_sum(27, 28))
    print(collatz_sum(5, 5))
    room = native.stack_alloc[int](4095)
    print(collatz_steps(room, 1, 4096))
    best = 0
    for i in range(4095):
        v = native.load(native.offset(room, i))
        if v > best:
            best = v
    print(best)
    print(native.load(native.offset(room, 26)))


main()
'''


def _ppy(reference: Path, cwd: Path, *args: str) -> str:
    env = dict(os.environ)
    env["PYTHONPATH"] = str(reference / "src")
    done = subprocess.run([sys.executable, "-m", "ppy_compiler", *args], cwd=cwd,
                          capture_output=True, text=True, env=env, check=False)
    if done.returncode != 0:
        raise RuntimeError(f"ppy {' '.join(args)} failed:\n{done.stdout}\n{done.stderr}")
    return done.stdout


def _with_collatz_max(text: str) -> str:
    """Add @collatz_collatz_max: collatz_sum's IR with the reduction's `op` and the body's
    fold made `max`. The frontend only turns `+=`/`*=` into parallel reductions, but the
    IR op takes add, mul, min and max (ir/dialects/parallel.py:31-32), so the max of the
    step counts is written here as IR, from the frontend's own sum."""
    from ppy_compiler.ir import decode, encode, verify

    start = text.index("func @collatz_collatz_sum(")
    end = text.index("\n}\n", start) + 3
    head = text[start:end]
    body_start = text.index("private func @collatz_collatz_sum__par1(")
    body_end = text.index("\n}\n", body_start) + 3
    body = text[body_start:body_end]
    head = (head.replace("@collatz_collatz_sum__par1", "@collatz_collatz_max__par1")
            .replace("@collatz_collatz_sum(", "@collatz_collatz_max(")
            .replace('op = "add"', 'op = "max"')
            .replace("collatz.collatz_sum", "collatz.collatz_max")
            .replace("ppy_collatz_collatz_sum", "ppy_collatz_collatz_max"))
    fold = "    %22 = core.add %20, %21 {overflow = \"python\"} : i64\n"
    assert body.count(fold) == 1
    body = (body.replace(fold, "    %22c = core.cmp.ge %20, %21 : bool\n"
                               "    %22 = core.select %22c, %20, %21 : i64\n")
            .replace("@collatz_collatz_sum__par1", "@collatz_collatz_max__par1")
            .replace("collatz_collatz_sum__par1", "collatz_collatz_max__par1"))
    combined = text.rstrip("\n") + "\n\n" + head + "\n" + body
    module = decode(combined)
    problems = verify(module)
    assert not problems, problems
    return encode(module)


PARALLEL_MATH = '''
import math

from ppy import native, parallel


def collatz_steps_of(n: int) -> int:
    x = n
    steps = 0
    while x != 1:
        if x % 2 == 0:
            x = x // 2
        else:
            x = 3 * x + 1
        steps += 1
    return steps


def math_table(out: native.ptr[float], lo: int, hi: int) -> int:
    for i in parallel.range(lo, hi):
        x = (i - 500) * 0.01
        native.store(native.offset(out, i - lo), math.tanh(x) + math.erf(x) + math.atan2(x, 1.5))
    return hi - lo


def asin_table(out: native.ptr[float], lo: int, hi: int) -> int:
    for i in parallel.range(lo, hi):
        native.store(native.offset(out, i - lo), math.asin(i * 0.25))
    return hi - lo
'''


def _with_collatz_map(text: str) -> str:
    """Add @pmath_collatz_map(out, lo, hi): `parallel.map @pmath_collatz_steps_of() lo, hi,
    out`, built with the reference's own builder (ir/dialects/parallel.py:184). The frontend
    never emits parallel.map (a loop that stores per index becomes parallel.for), so the
    op reaches a backend only from IR like this."""
    from ppy_compiler.ir import I64, Builder, PtrType, decode, encode, verify
    from ppy_compiler.ir.dialects import core, parallel

    module = decode(text)
    f = module.add_function("pmath_collatz_map",
                            [("out", PtrType(I64)), ("lo", I64), ("hi", I64)], [I64])
    f.attributes.update({"ppy.abi": "ppy", "ppy.symbol": "ppy_pmath_collatz_map",
                         "ppy.qualname": "pmath.collatz_map"})
    b = Builder(f.add_entry_block())
    out, lo, hi = f.entry.arguments
    parallel.map_(b, "pmath_collatz_steps_of", (), lo, hi, out)
    core.ret(b, core.sub(b, hi, lo))
    problems = verify(module)
    assert not problems, problems
    return encode(module)


def _call_ptr(engine, symbol, out: np.ndarray, lo: int, hi: int) -> tuple[int, int]:
    """Call a JIT'd function taking (ptr<T> out, i64 lo, i64 hi) and the result slot."""
    slot = ctypes.c_int64(0)
    fn = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                          ctypes.POINTER(ctypes.c_int64))(engine.address(symbol))
    return int(fn(out.ctypes.data, lo, hi, ctypes.byref(slot))), int(slot.value)


def golden_parallel_math(reference: Path) -> None:
    """parallel.map, and parallel.for bodies that call the math externs: the IR as the
    `openmp` route hands it to a backend (tests/golden/parallel_math.ppyir), and the outputs
    of the reference's LLVM JIT of that IR (parallel_math.npz): the Collatz step counts of
    [1, 5000) stored by the map at out[i], tanh(x) + erf(x) + atan2(x, 1.5) at x = (i -
    500) / 100 for i in [0, 1000) through ppy_math_unary/binary (src/ppy_runtime/stdlib.c:
    497-528), asin(i / 4) for i in [0, 5) (in its domain) and the status of [0, 8), where
    asin(1.25) fails the domain guard around the call (lowering/stdlib.py:693-731)."""
    from ppy_compiler.backend.llvm.from_ir import emit_module
    from ppy_compiler.backend.llvm.ir_pipeline import optimize
    from ppy_compiler.backend.llvm.jit import JitEngine
    from ppy_compiler.driver.config import ParallelConfig
    from ppy_compiler.ir import decode

    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        (root / "pyproject.toml").write_text(
            '[project]\nname = "pmath"\nversion = "0"\n\n[tool.ppy.parallel]\n'
            'backend = "openmp"\n', encoding="utf-8")
        (root / "pmath.ppy").write_text(textwrap.dedent(PARALLEL_MATH), encoding="utf-8")
        text = _with_collatz_map(_ppy(reference, root, "emit", "ir", "pmath.ppy"))
    (HERE / "parallel_math.ppyir").write_text(text, encoding="utf-8")
    module = decode(text)
    optimize(module, 2, parallel=ParallelConfig(backend="serial"))
    engine = JitEngine(opt_level=2).open()
    # ppy_math_unary/binary live in the reference's C runtime, which `ppy run` compiles into
    # its cache and loads into the JIT (backend/llvm/__init__.py:1052-1069): the same here,
    # with the cache in a temporary directory
    with tempfile.TemporaryDirectory() as cache:
        os.environ["XDG_CACHE_HOME"] = cache
        from ppy_runtime.collections import library_path

        runtime = library_path()
        assert runtime is not None, "the reference's C runtime did not build"
        engine.load_library(str(runtime))
    engine.add(emit_module(module))
    engine.finalize()
    steps = np.full(5000, -1, np.int64)
    map_status, map_value = _call_ptr(engine, "ppy_pmath_collatz_map", steps, 1, 5000)
    table = np.zeros(1000, np.float64)
    table_status, table_value = _call_ptr(engine, "ppy_pmath_math_table", table, 0, 1000)
    asin_ok = np.zeros(5, np.float64)
    asin_status, _ = _call_ptr(engine, "ppy_pmath_asin_table", asin_ok, 0, 5)
    asin_bad = np.zeros(8, np.float64)
    asin_bad_status, _ = _call_ptr(engine, "ppy_pmath_asin_table", asin_bad, 0, 8)
    np.savez_compressed(
        HERE / "parallel_math.npz", steps=steps, map_status=np.int32(map_status),
        map_value=np.int64(map_value), table=table, table_status=np.int32(table_status),
        table_value=np.int64(table_value), asin=asin_ok, asin_status=np.int32(asin_status),
        asin_bad_status=np.int32(asin_bad_status))


def golden_layernorm() -> None:
    """IR only: bf16 tensors are refused by the reference's LowerTensor; the parity of
    this module is checked against torch.layer_norm on the GPU."""
    write_ppyir(shared_passes(build_layernorm(), False), "gpt2_layernorm")


def golden_collatz_threads(reference: Path) -> None:
    """The same Collatz program as PPy's default `threads` route hands it to a backend:
    each `parallel.range` already split into host-thread chunks (`concurrency.spawn`)."""
    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        (root / "pyproject.toml").write_text('[project]\nname = "collatz"\nversion = "0"\n',
                                             encoding="utf-8")
        (root / "collatz.ppy").write_text(textwrap.dedent(COLLATZ), encoding="utf-8")
        text = _ppy(reference, root, "emit", "ir", "collatz.ppy")
        assert "concurrency.spawn" in text
        (HERE / "collatz_threads.ppyir").write_text(text, encoding="utf-8")


def golden_collatz(reference: Path) -> None:
    from ppy_compiler.ir import decode

    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        # The IR a backend receives: parallel.* kept intact by the openmp setting.
        (root / "pyproject.toml").write_text(
            '[project]\nname = "collatz"\nversion = "0"\n\n[tool.ppy.parallel]\n'
            'backend = "openmp"\n', encoding="utf-8")
        (root / "collatz.ppy").write_text(textwrap.dedent(COLLATZ), encoding="utf-8")
        text = _ppy(reference, root, "emit", "ir", "collatz.ppy")
        text = _with_collatz_max(text)
        (HERE / "collatz.ppyir").write_text(text, encoding="utf-8")
        # The reference's own answer: `ppy run` on the LLVM backend with threads.
        run_root = root / "run"
        run_root.mkdir()
        (run_root / "pyproject.toml").write_text(
            '[project]\nname = "collatzrun"\nversion = "0"\n', encoding="utf-8")
        (run_root / "collatz.ppy").write_text(
            textwrap.dedent(COLLATZ) + textwrap.dedent(COLLATZ_MAIN), encoding="utf-8")
        printed = _ppy(reference, run_root, "run", "collatz.ppy").split()
    # The JIT'd sum over a range whose 3x+1 overflows int64 takes the fallback.
    from ppy_compiler.backend.llvm.from_ir import emit_module
    from ppy_compiler.backend.llvm.jit import JitEngine
    from ppy_compiler.driver.config import ParallelConfig

    module = decode(text)
    from ppy_compiler.backend.llvm.ir_pipeline import optimize

    optimize(module, 2, parallel=ParallelConfig(backend="serial"))
    engine = JitEngine(opt_level=2).open()
    engine.add(emit_module(module))
    engine.finalize()
    symbol = next(f.attributes["ppy.symbol"] for f in module.functions.values()
                  if f.name.endswith("collatz_sum"))
    ok_status, ok_value = call(engine, symbol, 1, 1000)
    big = (1 << 62) + 1
    over_status, _ = call(engine, symbol, big, big + 4)
    max_symbol = next(f.attributes["ppy.symbol"] for f in module.functions.values()
                      if f.name.endswith("collatz_max"))
    max_4096 = call(engine, max_symbol, 1, 4096)
    max_65536 = call(engine, max_symbol, 1, 1 << 16)
    record = {
        "sum_1_65536": int(printed[0]),
        "sum_1_1000": int(printed[1]),
        "sum_27_28": int(printed[2]),
        "sum_5_5": int(printed[3]),
        "steps_count_1_4096": int(printed[4]),
        "max_1_4096": int(printed[5]),
        "steps_of_27": int(printed[6]),
        "jit_sum_1_1000": [ok_status, ok_value],
        "jit_overflow_status": over_status,
        "jit_max_1_4096": list(max_4096),
        "jit_max_1_65536": list(max_65536),
        "overflow_range": [big, big + 4],
    }
    (HERE / "collatz.json").write_text(json.dumps(record, indent=1) + "\n", encoding="utf-8")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, default=os.environ.get("PPY_REFERENCE"),
                        required="PPY_REFERENCE" not in os.environ,
                        help="a PPy checkout (default: $PPY_REFERENCE)")
    parser.add_argument("--only", help="write one fixture (e.g. views) and no other")
    options = parser.parse_args()
    _setup(options.reference)
    if options.only:
        make = globals()[f"golden_{options.only}"]
        make(options.reference) if make.__code__.co_argcount else make()
        print("golden fixture written to", HERE)
        return
    golden_chain()
    golden_gelu()
    golden_rows()
    golden_reductions()
    golden_matmul()
    golden_layernorm()
    golden_views()
    golden_collatz(options.reference)
    golden_collatz_threads(options.reference)
    golden_parallel_math(options.reference)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
