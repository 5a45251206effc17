"""The `b200_tensor` PPy plugin: a vocabulary for `ppy.Tensor` values in `.ppy` source.

`ppy.Tensor` has no arithmetic of its own in PPy (`a * b` on two of them is E1302); a plugin
has to type the operations, as the fixture plugin of the reference's
tests/test_common_tensor_lowering.py:69-149 does. This one claims the module
`ppy_b200.tensor` and answers each of its calls with the tensor-dialect operation it is
(`DialectOperationSpec("tensor", ...)`, plugins/base.py:121-135), so that PPy source reaches
the backend as the same tensor IR a `.ppyir` file holds:

    bt.add/sub/mul/div/pow/minimum/maximum(a, b)   tensor.<op>            (broadcasting)
    bt.exp/log/sqrt/... (x)                        tensor.unary {op}
    bt.sum/prod/max/min(x, axes=(..), keepdims=..) tensor.reduce {op, axes, keepdims}
    bt.matmul(a, b)                                tensor.matmul
    bt.convert(x, dtype="bf16")                    tensor.convert
    bt.full(value, dtype="f32")                    b200.fill      (a rank-0 tensor)
    bt.assign(out, value)                          b200.assign    (into a Mut tensor parameter)

The two `b200` operations exist because the tensor dialect has neither a typed scalar
broadcast from a Python float nor a write into a tensor parameter; the backend's first pass
(`ppy_b200.passes.CommonTensorsToBuffers`) rewrites them, and the tensor parameters, into
`tensor.fill`, `tensor.load` and `tensor.store` over buffers, which is what the backend builds.
The enabled plugin is named in the project: `[tool.ppy.plugins.b200_tensor]`.
"""

from __future__ import annotations

from ppy_compiler.analysis import types as T
from ppy_compiler.analysis.effects import Effect, EffectSet
from ppy_compiler.analysis.refinements import Facts
from ppy_compiler.ir import Dialect, OpSpec
from ppy_compiler.ir import shape as shapes
from ppy_compiler.ir.dialects import tensor as tensor_dialect
from ppy_compiler.plugins import CallArgument, CallResult, DialectOperationSpec, Plugin

from . import tensor as vocabulary

__all__ = ["B200Dialect", "TensorPlugin", "create_plugin"]

MODULE = "ppy_b200.tensor"
COMMON_TENSOR = T.Instance("ppy.Tensor", (), ("ppy.Tensor", "object"))

#: `dtype=` spellings and the names PPy's facts use for element types.
DTYPES = {"f32": "float32", "float32": "float32", "f64": "float64", "float64": "float64",
          "bf16": "bfloat16", "bfloat16": "bfloat16", "f16": "float16", "float16": "float16",
          "i32": "int32", "int32": "int32", "i64": "int64", "int64": "int64"}


def _verify_assign(op, checker) -> None:
    target = tensor_dialect.describe(op.operands[0].type)
    value = tensor_dialect.describe(op.operands[1].type)
    if target is None or value is None:
        checker.error(op, "b200.assign writes a tensor into a tensor parameter")
        return
    if target.dtype != value.dtype:
        checker.error(op, f"b200.assign of {value.dtype} into a tensor of {target.dtype}")
        return
    try:
        if shapes.broadcast(target.shape, value.shape) != tuple(target.shape):
            raise shapes.ShapeError(f"{value.shape} does not broadcast to {target.shape}")
    except shapes.ShapeError as error:
        checker.error(op, str(error))


def _verify_fill(op, checker) -> None:
    result = tensor_dialect.describe(op.results[0].type)
    if result is None or tuple(result.shape) != ():
        checker.error(op, "b200.fill gives a rank-0 tensor")


class B200Dialect(Dialect):
    """Two operations the tensor dialect lacks (see the module docstring)."""

    name = "b200"
    version = 1

    def register_operations(self, registry) -> None:
        registry.add_op(OpSpec("b200.assign", verify=_verify_assign, operands=2, results=0))
        registry.add_op(OpSpec("b200.fill", pure=True, verify=_verify_fill, operands=1,
                               results=1, required_attributes=("dtype",)))


def _tensor_facts(facts: Facts) -> tuple[str, tuple] | None:
    if facts.dtype is None or facts.shape is None:
        return None
    return facts.dtype, tuple(facts.shape)


def _result(dtype: str, shape: tuple, spec: DialectOperationSpec, count: int) -> CallResult:
    return CallResult(COMMON_TENSOR, Facts(dtype=dtype, shape=shape, ownership="owned"),
                      lowering=spec,
                      arguments=tuple(CallArgument(i, "borrowed") for i in range(count)))


class TensorPlugin(Plugin):
    name = "b200_tensor"
    modules = (MODULE,)

    def fingerprint(self) -> str:
        from . import __version__

        return f"api{self.api_version}:{self.name}:{__version__}"

    def register_dialects(self, registry) -> None:
        registry.register(B200Dialect())

    def call(self, qualname, args, keywords):
        if not qualname.startswith(MODULE + "."):
            return None
        name = qualname[len(MODULE) + 1:]
        tensors = [_tensor_facts(facts) for _type, facts in args]
        if name in vocabulary.BINARY and len(args) == 2 and None not in tensors:
            (da, sa), (db, sb) = tensors
            if da != db:
                return None
            try:
                shape = tuple(shapes.broadcast(sa, sb))
            except shapes.ShapeError:
                return None
            return _result(da, shape, DialectOperationSpec("tensor", vocabulary.BINARY[name]), 2)
        if name in vocabulary.UNARY and len(args) == 1 and tensors[0] is not None:
            dtype, shape = tensors[0]
            return _result(dtype, shape,
                           DialectOperationSpec("tensor", "unary", (("op", name),)), 1)
        if name in vocabulary.REDUCTIONS and len(args) == 1 and tensors[0] is not None:
            dtype, shape = tensors[0]
            axes = keywords.get("axes")
            keep = keywords.get("keepdims")
            axes_value = axes[1].constant if axes is not None and axes[1].has_constant else None
            keep_value = keep[1].constant if keep is not None and keep[1].has_constant else False
            if axes_value is None or not isinstance(keep_value, bool):
                return None
            try:
                reduced = tuple(shapes.reduce(shape, tuple(axes_value), keep_value))
            except shapes.ShapeError:
                return None
            spec = DialectOperationSpec("tensor", "reduce",
                                        (("op", vocabulary.REDUCTIONS[name]),),
                                        keyword_attributes=("axes", "keepdims"))
            return _result(dtype, reduced, spec, 1)
        if name == "matmul" and len(args) == 2 and None not in tensors:
            (da, sa), (db, sb) = tensors
            if da != db:
                return None
            try:
                shape = tuple(shapes.matmul(sa, sb))
            except shapes.ShapeError:
                return None
            return _result(da, shape, DialectOperationSpec("tensor", "matmul"), 2)
        if name == "convert" and len(args) == 1 and tensors[0] is not None:
            wanted = keywords.get("dtype")
            target = DTYPES.get(wanted[1].constant) if wanted is not None else None
            if target is None:
                return None
            spec = DialectOperationSpec("tensor", "convert", keyword_attributes=("dtype",))
            return _result(target, tensors[0][1], spec, 1)
        if name == "full" and len(args) == 1:
            wanted = keywords.get("dtype")
            if wanted is None:
                spec = DialectOperationSpec("b200", "fill", (("dtype", "f32"),))
                return _result("float32", (), spec, 1)
            target = DTYPES.get(wanted[1].constant)
            if target is None:
                return None
            spec = DialectOperationSpec("b200", "fill", keyword_attributes=("dtype",))
            return _result(target, (), spec, 1)
        if name == "assign" and len(args) == 2 and None not in tensors:
            return CallResult(T.NONE, effects=EffectSet.of(Effect.WRITE_MEMORY),
                              lowering=DialectOperationSpec("b200", "assign"),
                              arguments=(CallArgument(0, "mut"), CallArgument(1, "borrowed")))
        return None


def create_plugin(options=None) -> TensorPlugin:
    """The `ppy.plugins` entry point's factory."""
    return TensorPlugin(options)
