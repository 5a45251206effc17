"""`ppy.Tensor` operations for PPy source that targets the b200 backend.

In a `.ppy` module, `import ppy_b200.tensor as bt` and the `b200_tensor` plugin
(`ppy_b200.tensor_plugin`, enabled by `[tool.ppy.plugins.b200_tensor]` in the project) types
every call below into the tensor dialect, so that a function such as

    def gelu(a: ppy.Tensor[ppy.f32, (N,)], b: ..., c: ...,
             out: ppy.Mut[ppy.Tensor[ppy.f32, (N,)]]) -> None:
        z = bt.add(bt.mul(a, b), c)
        ...
        bt.assign(out, y)

reaches the backend as tensor operations that FuseTensor fuses and the backend builds into
kernels. Run by CPython, the same calls are these NumPy functions: the program's Python
meaning, element for element what the tensor dialect says (tensor.py:625-701 of the
reference: broadcasting binaries, NaN-propagating minimum/maximum, whole-axis reductions).
"""

from __future__ import annotations

import numpy as np

__all__ = ["BINARY", "UNARY", "REDUCTIONS", "add", "sub", "mul", "div", "pow", "minimum",
           "maximum", "sum", "prod", "max", "min", "matmul", "convert", "full", "assign"]

#: The elementwise binaries and the tensor dialect operation each is.
BINARY = {"add": "add", "sub": "sub", "mul": "mul", "div": "div", "pow": "pow",
          "minimum": "min", "maximum": "max"}
#: The reductions and the `tensor.reduce` op each is.
REDUCTIONS = {"sum": "add", "prod": "mul", "max": "max", "min": "min"}
#: The unary functions with their NumPy meaning (the names are `tensor.unary` ops).
UNARY = {"sqrt": np.sqrt, "sin": np.sin, "cos": np.cos, "tan": np.tan, "exp": np.exp,
         "exp2": np.exp2, "log": np.log, "log2": np.log2, "log10": np.log10,
         "floor": np.floor, "ceil": np.ceil, "trunc": np.trunc, "abs": np.abs,
         "neg": np.negative}


def add(a, b):
    return np.add(a, b)


def sub(a, b):
    return np.subtract(a, b)


def mul(a, b):
    return np.multiply(a, b)


def div(a, b):
    return np.divide(a, b)


def pow(a, b):  # noqa: A001 - the tensor dialect's name
    return np.power(a, b)


def minimum(a, b):
    return np.minimum(a, b)


def maximum(a, b):
    return np.maximum(a, b)


def _unary(name):
    fn = UNARY[name]

    def apply(x):
        return fn(x)

    apply.__name__ = name
    return apply


for _name in UNARY:
    globals()[_name] = _unary(_name)
    __all__.append(_name)


def _reduce(ufunc):
    def apply(x, axes=None, keepdims=False):
        return ufunc.reduce(x, axis=tuple(axes) if axes is not None else None,
                            keepdims=keepdims)

    return apply


sum = _reduce(np.add)  # noqa: A001
prod = _reduce(np.multiply)
max = _reduce(np.maximum)  # noqa: A001 - NaN-propagating, as tensor.reduce {op = "max"}
min = _reduce(np.minimum)  # noqa: A001


def matmul(a, b):
    return np.matmul(a, b)


_DTYPES = {"f32": np.float32, "f64": np.float64, "i32": np.int32, "i64": np.int64}


def convert(x, dtype="f32"):
    return np.asarray(x).astype(_DTYPES[dtype])


def full(value, dtype="f32"):
    """A rank-0 tensor holding `value`: broadcasts against any tensor of its element type."""
    return np.asarray(value, dtype=_DTYPES[dtype])


def assign(out, value):
    """The mutable tensor `out` takes `value` (broadcast to its shape)."""
    out[...] = value
