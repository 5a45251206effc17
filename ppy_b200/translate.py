"""Canonical IR -> kernel plan: what the b200 backend makes of a PPy module.

This is the only module of the backend that reads PPy's IR objects (it runs where
`ppy build` runs; the runtime never imports it). A function is one of:

* a **tensor function** -- one block of `tensor.*` / `linalg.matmul` operations on
  buffers, ending in `core.ret` of a constant (the shape every tensor module has after
  the shared passes, e.g. tests/golden/gelu.ppyir). Its operations are partitioned into
  kernels: maximal runs over one iteration space become one map kernel or one row
  kernel (a row kernel holds the reductions over the trailing axes that FuseTensor
  leaves as separate `tensor.reduce`/`tensor.fused` operations), whole-array and
  leading-axis reductions become two-pass reductions, and a matmul takes the
  elementwise group that follows it as its epilogue. Values crossing kernels become
  device temporaries; everything else stays in registers.
* a **scalar function** -- core arithmetic and control flow, possibly with
  `parallel.for/reduce/map` operations (what `ppy.parallel.range` lowers to under the
  `openmp` setting, ir/dialects/parallel.py:1-14). Its body becomes C++ (`scalar_c`),
  and each parallel operation a kernel over its range running the outlined body.

Anything else is refused with the reason, as `Backend.validate` must
(backend/base.py:255-258).
"""

from __future__ import annotations

from dataclasses import dataclass

from . import plan as P
from .scalar_c import ScalarEmitter, Unsupported

__all__ = ["Unsupported", "plan_module"]

#: Largest row a row kernel holds in registers (elements).
ROW_MAX_COLS = 8192


def _tensors():
    from ppy_compiler.ir.dialects import tensor as tensors

    return tensors


def dtype_name(t) -> str:
    text = str(t)
    if text not in P.CTYPES:
        raise Unsupported(f"elements of type {text}", "f32/f64/bf16/integer elements")
    return text


def _shape(info) -> tuple:
    from ppy_compiler.ir import shape as shapes

    dims = []
    for dim in info.shape:
        if isinstance(dim, int):
            dims.append(dim)
        elif isinstance(dim, shapes.Symbol):
            dims.append(dim.name)
        else:
            raise Unsupported(f"the dimension {shapes.spell(dim)}", "dimensions that are numbers or symbols")
    return tuple(dims)


def tensor_info(value):
    info = _tensors().describe(value.type)
    if info is None:
        return None
    if info.layout.strides is not None or info.layout.order != "row_major":
        raise Unsupported(f"a tensor with layout {value.type}", "row-major tensors")
    return info


def broadcast_shape(a: tuple, b: tuple) -> tuple:
    """NumPy's right-aligned broadcast of two shapes (symbols compare by name)."""
    rank = max(len(a), len(b))
    pa = (1,) * (rank - len(a)) + tuple(a)
    pb = (1,) * (rank - len(b)) + tuple(b)
    out = []
    for x, y in zip(pa, pb):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise Unsupported(f"shapes {a} and {b} that do not broadcast")
    return tuple(out)


# -- group formation -------------------------------------------------------------------


MAP_OPS = {"tensor.fused", "tensor.unary", "tensor.convert", "tensor.add", "tensor.sub",
           "tensor.mul", "tensor.div", "tensor.pow", "tensor.min", "tensor.max"}
VIEW_OPS = {"tensor.load", "tensor.fill", "tensor.broadcast", "tensor.reshape",
            "tensor.shape_cast", "tensor.transpose", "tensor.slice"}
#: Views onto memory that already exists, read through offsets and strides
#: (lower_tensor.py:695-714): a map reads them in place, other kernels from a copy.
STRIDED_OPS = ("tensor.transpose", "tensor.slice")
REDUCE_OPS = {"tensor.reduce"}
MATMUL_OPS = {"tensor.matmul", "linalg.matmul"}


def _reduce_of(op):
    """(kind, axes, keepdims) when `op` is a reduction, else None."""
    if op.name == "tensor.reduce":
        return str(op.attributes["op"]), tuple(int(a) for a in op.attributes["axes"]), bool(
            op.attributes.get("keepdims", False))
    if op.name == "tensor.fused" and op.attributes.get("reduce") is not None:
        return str(op.attributes["reduce"]), tuple(int(a) for a in op.attributes["axes"]), bool(
            op.attributes.get("keepdims", False))
    return None


@dataclass
class _Group:
    kind: str  # "map" | "row" | "reduce_all" | "reduce_cols" | "matmul"
    frame: tuple
    reduced: int = 0
    ops: list = None  # type: ignore[assignment]

    def __post_init__(self) -> None:
        if self.ops is None:
            self.ops = []


def _row_shape(frame: tuple, reduced: int) -> tuple:
    return tuple(frame[: len(frame) - reduced])


class _TensorTranslator:
    def __init__(self, module, function, symbol: str) -> None:
        self.module = module
        self.function = function
        self.symbol = symbol
        self.counter = 0
        self.params: list[P.Param] = []
        self.param_by_value: dict[int, P.Param] = {}
        self.bindings: list[P.Binding] = []
        self.bound: set[str] = set()
        self.guards: list = []
        self.temps: list[P.Temp] = []
        self.kernels: list = []
        self.values: dict[int, tuple] = {}  # id(value) -> ("param", Param) | ("temp", Temp)
        #: transposes/slices copied to a contiguous temporary for a kernel that reads rows
        self.materialized: set[int] = set()
        self.dim_guards: list = []

    def fresh(self, hint: str) -> str:
        self.counter += 1
        return f"{hint}{self.counter}"

    # ---------------------------------------------------------------- entry

    def run(self) -> P.TensorFunction:
        fn = self.function
        blocks = fn.body.blocks
        if len(blocks) != 1:
            raise Unsupported(f"@{fn.name}: a tensor function with control flow",
                              "one block of tensor operations")
        for (name, t), argument in zip(fn.params, fn.entry.arguments):
            text = str(t)
            if text.startswith("buffer<"):
                param = P.Param(name, "buffer", dtype_name(t.element))
            elif text.startswith("ptr<"):
                raise Unsupported(f"@{fn.name}: pointer parameter {name} of a tensor function",
                                  "buffer parameters")
            else:
                param = P.Param(name, "scalar", dtype_name(t))
            self.params.append(param)
            self.param_by_value[id(argument)] = param
        ops = list(blocks[0].operations)
        terminator = ops[-1]
        if terminator.name != "core.ret":
            raise Unsupported(f"@{fn.name}: a block ending in {terminator.name}")
        result, result_value = self._result(terminator)
        body = ops[:-1]
        for op in body:
            if op.dialect not in ("tensor", "linalg", "core"):
                raise Unsupported(f"@{fn.name}: {op.name} in a tensor function")
            if op.dialect == "core" and op.name != "core.const":
                raise Unsupported(f"@{fn.name}: {op.name} among tensor operations",
                                  "tensor functions of tensor operations and constants")
        self._bind(body)
        groups = self._partition(body)
        self._materialize(body, groups)
        for group in groups:
            kernel = self._kernel(group)
            self.kernels.extend(kernel if isinstance(kernel, list) else [kernel])
        for param in self.params:
            if param.kind == "buffer":
                reads, writes = bool(param.read_shapes), bool(param.write_shapes)
                param.role = "inout" if reads and writes else "in" if reads else (
                    "out" if writes else "")
        return P.TensorFunction(fn.name, self.symbol, self.params, result, result_value,
                                self.bindings, self.guards, self.temps, self.kernels,
                                dim_guards=self.dim_guards)

    def _result(self, ret):
        if not ret.operands:
            return None, 0
        if len(ret.operands) != 1:
            raise Unsupported(f"@{self.function.name}: several results")
        value = ret.operands[0]
        owner = value.owner
        if owner is None or getattr(owner, "name", None) != "core.const":
            raise Unsupported(f"@{self.function.name}: a result computed from tensors",
                              "tensor functions returning a constant")
        return dtype_name(value.type), int(owner.attributes["value"])

    # ---------------------------------------------------------------- symbols and guards

    def _bind(self, body) -> None:
        """Bind symbolic dimensions where loads name them (lower_tensor.py:233-277)."""
        for op in body:
            if op.name == "tensor.load":
                buffer = self.param_by_value.get(id(op.operands[0]))
                if buffer is None:
                    raise Unsupported("a load from something other than a parameter")
                shape = _shape(tensor_info(op.result))
                unknown = sorted({d for d in shape if isinstance(d, str)} - self.bound)
                if len(unknown) > 1:
                    raise Unsupported(f"@{self.function.name}: {shape} has {len(unknown)} "
                                      "unknown dimensions; one buffer length binds one")
                if unknown:
                    name = unknown[0]
                    if shape.count(name) != 1:
                        raise Unsupported(f"@{self.function.name}: {name} in {shape} cannot be "
                                          "read from a buffer length")
                    rest = tuple(d for d in shape if d != name)
                    self.bindings.append(P.Binding(name, buffer.name, rest))
                    self.bound.add(name)
                self.guards.append((buffer.name, shape))
                buffer.read_shapes.append(shape)
            elif op.name == "tensor.store":
                buffer = self.param_by_value.get(id(op.operands[1]))
                if buffer is None:
                    raise Unsupported("a store into something other than a parameter")
                shape = self._known(_shape(tensor_info(op.operands[0])))
                self.guards.append((buffer.name, shape))
                buffer.write_shapes.append(shape)
            else:
                for result in op.results:
                    info = tensor_info(result)
                    if info is not None:
                        self._known(_shape(info))

    def _known(self, shape: tuple) -> tuple:
        for dim in shape:
            if isinstance(dim, str) and dim not in self.bound:
                raise Unsupported(f"@{self.function.name}: dimension {dim} is not bound; "
                                  "load a tensor whose shape names it first")
        return shape

    # ---------------------------------------------------------------- partition

    def _partition(self, body) -> list[_Group]:
        groups: list[_Group] = []
        current: _Group | None = None
        # Converts that feed a matmul are read by the matmul kernel itself.
        absorbed = set()
        for op in body:
            if op.name in MATMUL_OPS:
                for operand in op.operands:
                    owner = operand.owner
                    if getattr(owner, "name", None) == "tensor.convert" and all(
                        user is op for user, _ in operand.uses
                    ):
                        absorbed.add(id(owner))
        self._decide_copies(body)
        for op in body:
            if op.name in STRIDED_OPS and id(op.results[0]) in self.materialized:
                current = None
                value = op.results[0]
                groups.append(_Group("map", _shape(tensor_info(value)), ops=[("copy", value)]))
                continue
            if op.name in VIEW_OPS or op.name == "core.const" or op.name == "tensor.store":
                continue
            if id(op) in absorbed:
                continue
            if op.name == "tensor.concat":
                current = None
                groups.append(_Group("concat", _shape(tensor_info(op.results[0])), ops=[op]))
                continue
            if op.name in MATMUL_OPS:
                current = None
                groups.append(_Group("matmul", _shape(tensor_info(op.result)), ops=[op]))
                continue
            reduction = _reduce_of(op)
            if reduction is not None:
                kind, axes, _keep = reduction
                source = self._frame_of(op)
                rank = len(source)
                if not axes:
                    raise Unsupported("a reduction over no axes")
                trailing = tuple(range(rank - len(axes), rank))
                if tuple(sorted(axes)) == tuple(range(rank)):
                    current = None
                    groups.append(_Group("reduce_all", source, rank, ops=[op]))
                    continue
                if tuple(sorted(axes)) == trailing:
                    cols = 1
                    static = True
                    for dim in source[rank - len(axes):]:
                        if isinstance(dim, int):
                            cols *= dim
                        else:
                            static = False
                    if static and cols <= ROW_MAX_COLS:
                        if current is not None and current.kind in ("map", "row") and (
                            current.frame == source
                            and (current.kind == "map" or current.reduced == len(axes))
                        ):
                            current.kind = "row"
                            current.reduced = len(axes)
                            current.ops.append(op)
                        else:
                            current = _Group("row", source, len(axes), ops=[op])
                            groups.append(current)
                        continue
                    raise Unsupported(f"a reduction over trailing axes of {source} with rows "
                                      f"longer than {ROW_MAX_COLS} or symbolic",
                                      "rows of at most 8192 static elements")
                if tuple(sorted(axes)) == tuple(range(len(axes))):
                    current = None
                    groups.append(_Group("reduce_cols", source, len(axes), ops=[op]))
                    continue
                raise Unsupported(f"a reduction over axes {axes} of {source}",
                                  "reductions over all, leading, or trailing axes")
            if op.name in MAP_OPS:
                shape = _shape(tensor_info(op.result))
                if current is not None and current.kind == "map" and current.frame == shape:
                    current.ops.append(op)
                    continue
                if current is not None and current.kind == "row" and not self._reads_view(op) and (
                    shape == current.frame
                    or self._is_rowwise(shape, current.frame, current.reduced)
                ):
                    current.ops.append(op)
                    continue
                current = _Group("map", shape, ops=[op])
                groups.append(current)
                continue
            raise Unsupported(f"{op.name}", "the tensor operations of the b200 backend")
        # A stored value no group computes (a loaded or filled tensor) is copied by a map.
        computed = {id(r) for g in groups for op in g.ops
                    for r in ([op[1]] if isinstance(op, tuple) else op.results)}
        for op in body:
            if op.name == "tensor.store" and id(op.operands[0]) not in computed:
                value = op.operands[0]
                groups.append(_Group("map", _shape(tensor_info(value)), ops=[("copy", value)]))
        return self._fuse_epilogues(groups)

    # ---------------------------------------------------------------- strided views

    def _decide_copies(self, body) -> None:
        """Transposes and slices that a row, reduction or matmul kernel reads (those read rows
        of contiguous memory) are copied to a temporary first; maps read them in place."""
        for op in body:
            if op.name not in STRIDED_OPS:
                continue
            value = op.results[0]
            for user, _ in value.uses:
                name = getattr(user, "name", None)
                feeds_matmul = name == "tensor.convert" and any(
                    getattr(u, "name", None) in MATMUL_OPS for u, _ in user.results[0].uses)
                if (_reduce_of(user) is not None or name in MATMUL_OPS or feeds_matmul
                        or name == "tensor.reshape"):
                    self.materialized.add(id(value))

    def _reads_view(self, op) -> bool:
        """Whether `op` reads a transpose or slice in place (through broadcasts)."""
        for operand in op.operands:
            value = operand
            while True:
                owner = value.owner
                name = getattr(owner, "name", None)
                if name in STRIDED_OPS:
                    if id(value) not in self.materialized:
                        return True
                    break
                if name in ("tensor.broadcast", "tensor.shape_cast", "tensor.reshape"):
                    value = owner.operands[0]
                    continue
                break
        return False

    def _strided(self, value, own: bool = False):
        """(base, offset, strides) when `value` is a transpose or slice (through any chain of
        views) read in place, else None: element (i0, i1, ...) of `value` is element
        offset + sum(i_k * strides[k]) of the memory of `base` (lower_tensor.py:695-714).
        `own` reads `value` itself in place even where it is copied (the copy's own read)."""
        owner = value.owner
        name = getattr(owner, "name", None)
        if name not in STRIDED_OPS or (id(value) in self.materialized and not own):
            return None
        source = owner.operands[0]
        base, offset, strides = self._memory_of(source)
        if name == "tensor.transpose":
            perm = tuple(int(p) for p in owner.attributes["perm"])
            return base, offset, tuple(strides[p] for p in perm)
        starts = tuple(int(v) for v in owner.attributes["starts"])
        stops = tuple(int(v) for v in owner.attributes["stops"])
        steps = tuple(int(v) for v in owner.attributes["steps"])
        for dim, stop in zip(_shape(tensor_info(source)), stops):
            # a slice that stops inside a symbolic dimension needs that much of it
            if isinstance(dim, str) and stop > 0 and (dim, stop) not in self.dim_guards:
                self.dim_guards.append((dim, stop))
        for start, stride in zip(starts, strides):
            offset = P.term_add(offset, P.term_mul(start, stride))
        return base, offset, tuple(P.term_mul(st, step) for st, step in zip(strides, steps))

    def _memory_of(self, value):
        """(base, offset, strides) of `value` as memory: a view's, or its own row-major
        layout (through broadcasts, which give stride 0 on the axes they add or widen)."""
        found = self._strided(value)
        if found is not None:
            return found
        owner = value.owner
        name = getattr(owner, "name", None)
        shape = _shape(tensor_info(value))
        if name in ("tensor.broadcast", "tensor.shape_cast"):
            inner = owner.operands[0]
            base, offset, strides = self._memory_of(inner)
            inner_shape = _shape(tensor_info(inner))
            if name == "tensor.shape_cast" or len(inner_shape) > len(shape):
                if self._strided(inner) is not None:
                    raise Unsupported("a shape cast of a transposed or sliced tensor",
                                      "transposes and slices of row-major tensors")
                return base, offset, P.contiguous_strides(shape)
            pad = len(shape) - len(inner_shape)
            out = []
            for d, dim in enumerate(shape):
                j = d - pad
                out.append(0 if j < 0 or (inner_shape[j] == 1 and dim != 1) else strides[j])
            return base, offset, tuple(out)
        if name == "tensor.reshape":
            inner = owner.operands[0]
            if self._strided(inner) is not None:
                raise Unsupported("a reshape of a transposed or sliced tensor",
                                  "reshapes of row-major tensors")
            base, offset, _ = self._memory_of(inner)
            return base, offset, P.contiguous_strides(shape)
        return value, 0, P.contiguous_strides(shape)

    def _frame_of(self, op) -> tuple:
        """The iteration shape of a reduction: its input's (broadcast) shape."""
        shape: tuple = ()
        for operand in op.operands:
            info = tensor_info(operand)
            if info is not None:
                shape = broadcast_shape(shape, _shape(info))
        return shape

    @staticmethod
    def _is_rowwise(shape: tuple, frame: tuple, reduced: int) -> bool:
        rows = _row_shape(frame, reduced)
        return shape == rows + (1,) * reduced or shape == rows

    def _fuse_epilogues(self, groups: list[_Group]) -> list[_Group]:
        """A matmul whose product only the next map group reads takes that group."""
        out: list[_Group] = []
        index = 0
        while index < len(groups):
            group = groups[index]
            nxt = groups[index + 1] if index + 1 < len(groups) else None
            if group.kind == "matmul" and nxt is not None and nxt.kind == "map" and (
                nxt.frame == group.frame
            ) and not any(not isinstance(op, tuple) and self._reads_view(op) for op in nxt.ops):
                product = group.ops[0].results[0]
                members = {id(op) for op in nxt.ops if not isinstance(op, tuple)}
                users = [user for user, _ in product.uses]
                if users and all(id(u) in members for u in users):
                    group.ops.extend(nxt.ops)
                    out.append(group)
                    index += 2
                    continue
            out.append(group)
            index += 1
        return out

    # ---------------------------------------------------------------- materialization

    def _materialize(self, body, groups: list[_Group]) -> None:
        """Decide where each group's results go: stored buffers and temporaries."""
        owner_group: dict[int, int] = {}
        for gi, group in enumerate(groups):
            for op in group.ops:
                if isinstance(op, tuple):
                    if getattr(op[1].owner, "name", None) in STRIDED_OPS:
                        owner_group[id(op[1])] = gi  # a view's copy
                    continue
                for result in op.results:
                    owner_group[id(result)] = gi
        self.stores: dict[int, list] = {}
        for op in body:
            if op.name == "tensor.store":
                param = self.param_by_value[id(op.operands[1])]
                self.stores.setdefault(id(op.operands[0]), []).append(param)
        self.crossing: set[int] = set()
        for gi, group in enumerate(groups):
            for op in group.ops:
                operands = [op[1]] if isinstance(op, tuple) else op.operands
                if isinstance(op, tuple) and getattr(op[1].owner, "name", None) in STRIDED_OPS:
                    operands = [op[1].owner.operands[0]]  # a view's copy reads its source
                for operand in operands:
                    source = self._through_views(operand)
                    og = owner_group.get(id(source))
                    if og is not None and og != gi:
                        self.crossing.add(id(source))
        for value_id in self.crossing:
            pass
        self.owner_group = owner_group

    def _through_views(self, value):
        """The value whose memory a view chain reads (broadcast/reshape/shape_cast, and
        transposes and slices read in place)."""
        while True:
            owner = value.owner
            name = getattr(owner, "name", None)
            if name in ("tensor.broadcast", "tensor.reshape", "tensor.shape_cast") or (
                    name in STRIDED_OPS and id(value) not in self.materialized):
                value = owner.operands[0]
                continue
            return value

    def _temp_for(self, value) -> P.Temp:
        found = self.values.get(id(value))
        if found is not None:
            return found[1]
        info = tensor_info(value)
        temp = P.Temp(self.fresh("tmp"), dtype_name(info.dtype), _shape(info))
        self.temps.append(temp)
        self.values[id(value)] = ("temp", temp)
        return temp

    # ---------------------------------------------------------------- kernels

    def _concat_kernels(self, group: _Group) -> list:
        """`tensor.concat` (lower_tensor.py:716-730): one copy per part into the result's
        memory at the part's position along the axis (the stored buffer and/or a temporary)."""
        op = group.ops[0]
        result = op.results[0]
        info = tensor_info(result)
        shape, dtype = _shape(info), dtype_name(info.dtype)
        axis = int(op.attributes["axis"])
        strides = P.contiguous_strides(shape)
        destinations = [("param", p.name, p.dtype) for p in self.stores.get(id(result), [])]
        if id(result) in self.crossing:
            temp = self._temp_for(result)
            destinations.append(("temp", temp.name, dtype))
        kernels, position = [], 0
        for k, part in enumerate(op.operands):
            pshape = _shape(tensor_info(part))
            builder = _ProgramBuilder(self, _Group("map", pshape, ops=[("copy", part)]))
            builder.build()
            var = builder.var_of[id(part)]
            view = (P.term_mul(position, strides[axis]), strides)
            outputs = [P.Output(var, P.Operand(source, name, dt, pshape, view=view))
                       for source, name, dt in destinations]
            kernels.append(P.MapKernel(f"{self.symbol}_k{len(self.kernels)}_{k}", pshape,
                                       builder.inputs, builder.program, outputs))
            position = P.term_add(position, P.dim_term(pshape[axis]))
        return kernels

    def _kernel(self, group: _Group):
        if group.kind == "concat":
            return self._concat_kernels(group)
        builder = _ProgramBuilder(self, group)
        name = f"{self.symbol}_k{len(self.kernels)}"
        if group.kind == "matmul":
            return builder.matmul(name)
        builder.build()
        outputs = builder.outputs()
        if group.kind == "map":
            return P.MapKernel(name, group.frame, builder.inputs, builder.program, outputs)
        if group.kind == "row":
            cols = 1
            for dim in group.frame[len(group.frame) - group.reduced:]:
                cols *= int(dim)
            return P.RowKernel(name, group.frame, group.reduced, cols, builder.inputs,
                               builder.program, outputs)
        root = group.ops[-1]
        var = builder.var_of[id(root.results[0])]
        reduce_stmt = next(s for s in builder.program if s.var == var)
        # The fold itself is the kernel's; the program yields the element it folds.
        builder.program.remove(reduce_stmt)
        if len(outputs) != 1:
            raise Unsupported("a whole-array reduction read by other operations",
                              "reductions whose result is stored")
        cls = P.ReduceAllKernel if group.kind == "reduce_all" else P.ReduceColsKernel
        if cls is P.ReduceAllKernel:
            return cls(name, group.frame, builder.inputs, builder.program, reduce_stmt.args[0],
                       reduce_stmt.attrs["kind"], reduce_stmt.dtype, outputs[0].operand)
        return cls(name, group.frame, group.reduced, builder.inputs, builder.program,
                   reduce_stmt.args[0], reduce_stmt.attrs["kind"], reduce_stmt.dtype,
                   outputs[0].operand)


class _ProgramBuilder:
    """Inline one group's operations into a scalar element program."""

    def __init__(self, owner: _TensorTranslator, group: _Group) -> None:
        self.owner = owner
        self.group = group
        self.inputs: list[P.Operand] = []
        self.input_index: dict[tuple, int] = {}
        self.program: list[P.Stmt] = []
        self.var_of: dict[int, str] = {}
        self.scalar_var: dict[int, str] = {}
        self.members = {id(op) for op in group.ops if not isinstance(op, tuple)}

    def fresh(self, hint: str = "v") -> str:
        self.owner.counter += 1
        return f"{hint}{self.owner.counter}"

    def emit(self, op: str, args: tuple, dtype: str, **attrs) -> str:
        var = self.fresh()
        self.program.append(P.Stmt(var, op, tuple(args), dtype, dict(attrs)))
        return var

    # ---------------------------------------------------------------- leaves

    def scalar(self, value) -> str:
        """A scalar operand: a constant or a scalar parameter."""
        found = self.scalar_var.get(id(value))
        if found is not None:
            return found
        owner = value.owner
        dtype = dtype_name(value.type)
        if getattr(owner, "name", None) == "core.const":
            var = self.emit("const", (), dtype, value=owner.attributes["value"])
        else:
            param = self.owner.param_by_value.get(id(value))
            if param is None:
                raise Unsupported("a scalar operand computed outside the group",
                                  "constants and scalar parameters")
            var = self.emit("param", (), dtype, name=param.name)
        self.scalar_var[id(value)] = var
        return var

    def tensor(self, value) -> str:
        """The element variable of tensor `value` inside this group."""
        if id(value) in self.var_of:
            return self.var_of[id(value)]
        owner = value.owner
        name = getattr(owner, "name", None)
        if name == "tensor.fill":
            return self.scalar(owner.operands[0])
        if name in ("tensor.broadcast", "tensor.shape_cast"):
            source = self.tensor_leaf(owner.operands[0], _shape(tensor_info(owner.operands[0])))
            return source
        if name == "tensor.reshape":
            return self.tensor_leaf(owner.operands[0], _shape(tensor_info(value)))
        return self.tensor_leaf(value, _shape(tensor_info(value)))

    def tensor_leaf(self, value, shape: tuple) -> str:
        """A tensor read from memory: a loaded parameter or another kernel's temporary,
        possibly through a strided view."""
        owner = value.owner
        name = getattr(owner, "name", None)
        if name == "tensor.fill":
            return self.scalar(owner.operands[0])
        if name in STRIDED_OPS:
            copying = any(isinstance(op, tuple) and op[1] is value for op in self.group.ops)
            if copying or id(value) not in self.owner.materialized:
                return self.view_leaf(value, shape, copying)
        if name in ("tensor.broadcast", "tensor.shape_cast", "tensor.reshape"):
            inner_shape = shape if name == "tensor.reshape" else _shape(tensor_info(owner.operands[0]))
            if name == "tensor.reshape":
                return self.tensor_leaf(owner.operands[0], shape)
            return self.tensor_leaf(owner.operands[0], inner_shape)
        if name == "tensor.load":
            param = self.owner.param_by_value[id(owner.operands[0])]
            operand = P.Operand("param", param.name, param.dtype, shape)
        elif id(value) in self.var_of:
            return self.var_of[id(value)]
        else:
            temp = self.owner._temp_for(value)
            operand = P.Operand("temp", temp.name, temp.dtype, shape)
        key = (operand.source, operand.name, operand.shape)
        index = self.input_index.get(key)
        if index is None:
            index = len(self.inputs)
            self.inputs.append(operand)
            self.input_index[key] = index
        return self.emit("input", (index,), operand.dtype)

    def view_leaf(self, value, shape: tuple, own: bool) -> str:
        """A transpose or slice read in place: its base memory with an offset and strides."""
        view_shape = _shape(tensor_info(value))
        if tuple(shape) != tuple(view_shape):
            raise Unsupported("a reshape of a transposed or sliced tensor",
                              "reshapes of row-major tensors")
        base, offset, strides = self.owner._strided(value, own=own)
        bowner = base.owner
        bname = getattr(bowner, "name", None)
        if bname == "tensor.fill":
            return self.scalar(bowner.operands[0])
        if bname == "tensor.load":
            param = self.owner.param_by_value[id(bowner.operands[0])]
            operand = P.Operand("param", param.name, param.dtype, view_shape, (offset, strides))
        else:
            temp = self.owner._temp_for(base)
            operand = P.Operand("temp", temp.name, temp.dtype, view_shape, (offset, strides))
        key = (operand.source, operand.name, operand.shape, operand.view)
        index = self.input_index.get(key)
        if index is None:
            index = len(self.inputs)
            self.inputs.append(operand)
            self.input_index[key] = index
        return self.emit("input", (index,), operand.dtype)

    # ---------------------------------------------------------------- operations

    def build(self) -> None:
        for op in self.group.ops:
            if isinstance(op, tuple):  # ("copy", value): a stored tensor no group computes
                value = op[1]
                self.var_of[id(value)] = self.tensor(value)
                continue
            self.var_of[id(op.results[0])] = self.lower(op)

    def lower(self, op) -> str:
        name = op.name
        if name == "tensor.fused":
            return self.fused(op)
        if name == "tensor.reduce":
            kind = str(op.attributes["op"])
            element = self.tensor(op.operands[0])
            dtype = dtype_name(tensor_info(op.result).dtype)
            return self.emit("reduce", (element,), dtype, kind=kind)
        if name == "tensor.unary":
            return self.unary(str(op.attributes["op"]), self.tensor(op.operands[0]),
                              dtype_name(tensor_info(op.result).dtype))
        if name == "tensor.convert":
            source = self.tensor(op.operands[0])
            return self.emit("cast", (source,), dtype_name(tensor_info(op.result).dtype))
        local = name.split(".", 1)[1]
        left = self.tensor(op.operands[0])
        right = self.tensor(op.operands[1])
        return self.binary(local, left, right, dtype_name(tensor_info(op.result).dtype))

    def binary(self, name: str, left: str, right: str, dtype: str) -> str:
        """`tensor.scalar_binary` (ir/dialects/tensor.py:667-682)."""
        if name in ("min", "max"):
            return self.extremum(name, left, right, dtype)
        if name == "pow":
            return self.emit("pow", (left, right), dtype)
        overflow = None if P.is_float(dtype) or name == "div" else "wrap"
        attrs = {"overflow": overflow} if overflow else {}
        if name == "div" and not P.is_float(dtype):
            attrs = {"rounding": "floor", "overflow": "python"}
        return self.emit(name, (left, right), dtype, **attrs)

    def extremum(self, kind: str, a: str, c: str, dtype: str) -> str:
        """`tensor.scalar_extremum` (ir/dialects/tensor.py:684-701): NaN-propagating."""
        keep = self.emit("cmp", (a, c), "bool", predicate="le" if kind == "min" else "ge")
        chosen = self.emit("select", (keep, a, c), dtype)
        if not P.is_float(dtype):
            return chosen
        number = self.emit("cmp", (a, a), "bool", predicate="eq")
        return self.emit("select", (number, chosen, a), dtype)

    def unary(self, kind: str, value: str, dtype: str) -> str:
        """`tensor.scalar_unary` (ir/dialects/tensor.py:653-665)."""
        if kind == "neg":
            return self.emit("neg", (value,), dtype, **({} if P.is_float(dtype) else {"overflow": "wrap"}))
        if kind == "abs" and not P.is_float(dtype):
            zero = self.emit("const", (), dtype, value=0)
            negative = self.emit("cmp", (value, zero), "bool", predicate="lt")
            flipped = self.emit("neg", (value,), dtype, overflow="wrap")
            return self.emit("select", (negative, flipped, value), dtype)
        from ppy_compiler.ir.dialects.math import UNARY as MATH_UNARY

        if kind in MATH_UNARY:
            return self.emit("math", (value,), dtype, fn=kind)
        return self.emit("special", (value,), dtype, fn=kind)

    def fused(self, op) -> str:
        body = op.regions[0].blocks[0]
        mapping: dict[int, str] = {}
        for argument, operand in zip(body.arguments, op.operands):
            if tensor_info(operand) is not None:
                mapping[id(argument)] = self.tensor(operand)
            else:
                mapping[id(argument)] = self.scalar(operand)
        produced = None
        for inner in body.operations:
            if inner.name == "tensor.yield":
                produced = mapping.get(id(inner.operands[0])) or self._outer(inner.operands[0])
                break
            args = tuple(mapping.get(id(v)) or self._outer(v) for v in inner.operands)
            mapping[id(inner.results[0])] = self.body_op(inner, args)
        assert produced is not None
        reduction = _reduce_of(op)
        if reduction is not None:
            dtype = dtype_name(tensor_info(op.result).dtype)
            return self.emit("reduce", (produced,), dtype, kind=reduction[0])
        return produced

    def _outer(self, value) -> str:
        return self.scalar(value)

    def body_op(self, inner, args: tuple) -> str:
        """One scalar operation of a fused body (core, math, special dialects)."""
        dtype = dtype_name(inner.results[0].type)
        name = inner.name
        dialect, local = name.split(".", 1)
        attrs = dict(inner.attributes)
        if dialect == "core":
            if local == "const":
                return self.emit("const", (), dtype, value=attrs["value"])
            if local in ("add", "sub", "mul", "div", "mod", "neg"):
                keep = {k: attrs[k] for k in ("overflow", "rounding") if k in attrs}
                return self.emit(local, args, dtype, **keep)
            if local in ("and", "or", "xor", "shl", "shr", "select", "cast"):
                return self.emit(local, args, dtype)
            if local == "cmp":
                return self.emit("cmp", args, "bool", predicate=str(attrs["predicate"]))
            raise Unsupported(f"{name} in a fused body")
        if dialect == "math":
            if local == "pow":
                return self.emit("pow", args, dtype)
            return self.emit("math", args, dtype, fn=local)
        if dialect == "special":
            return self.emit("special", args, dtype, fn=local)
        raise Unsupported(f"{name} in a fused body")

    # ---------------------------------------------------------------- outputs

    def outputs(self) -> list[P.Output]:
        result: list[P.Output] = []
        seen = set()
        for op in self.group.ops:
            values = [op[1]] if isinstance(op, tuple) else op.results
            for value in values:
                if id(value) in seen:
                    continue
                seen.add(id(value))
                var = self.var_of.get(id(value))
                if var is None:
                    continue
                info = tensor_info(value)
                shape = _shape(info)
                dtype = dtype_name(info.dtype)
                for param in self.owner.stores.get(id(value), []):
                    result.append(P.Output(var, P.Operand("param", param.name, param.dtype, shape)))
                if id(value) in self.owner.crossing:
                    temp = self.owner._temp_for(value)
                    result.append(P.Output(var, P.Operand("temp", temp.name, dtype, shape)))
        return result

    # ---------------------------------------------------------------- matmul

    def matmul(self, name: str) -> P.MatmulKernel:
        op = self.group.ops[0]
        a_value, b_value = op.operands

        def source(value):
            owner = value.owner
            if getattr(owner, "name", None) == "tensor.convert":
                value = owner.operands[0]
            info = tensor_info(value)
            shape = _shape(info)
            dtype = dtype_name(info.dtype)
            producer = value.owner
            if getattr(producer, "name", None) == "tensor.load":
                param = self.owner.param_by_value[id(producer.operands[0])]
                return P.Operand("param", param.name, dtype, shape)
            temp = self.owner._temp_for(value)
            return P.Operand("temp", temp.name, dtype, shape)

        a = source(a_value)
        b = source(b_value)
        if len(a.shape) != 2 or len(b.shape) != 2:
            raise Unsupported("a matmul of tensors that are not matrices", "rank-2 matmul")
        if a.dtype != b.dtype or a.dtype not in ("bf16", "f32"):
            raise Unsupported(f"a matmul of {a.dtype} by {b.dtype}", "bf16 or f32 operands")
        if not isinstance(a.shape[1], int) or not isinstance(b.shape[1], int):
            raise Unsupported("a matmul with a symbolic K or N", "static K and N")
        result_dtype = dtype_name(tensor_info(op.result).dtype)
        if result_dtype != "f32":
            raise Unsupported(f"a matmul giving {result_dtype}",
                              "f32 results (convert bf16 operands to f32 first)")
        # The epilogue program: input 0 is the product's element.
        product = P.Operand("temp", "__acc", "f32", (a.shape[0], b.shape[1]))
        self.inputs.append(product)
        self.input_index[("temp", "__acc", product.shape)] = 0
        acc = self.emit("input", (0,), "f32")
        self.var_of[id(op.results[0])] = acc
        for other in self.group.ops[1:]:
            self.var_of[id(other.results[0])] = self.lower(other)
        outputs = self.outputs()
        return P.MatmulKernel(name, a, b, a.shape[0], int(b.shape[1]), int(a.shape[1]),
                              self.inputs, self.program, outputs)


# -- module ----------------------------------------------------------------------------


def _symbol_of(function) -> str:
    symbol = function.attributes.get("ppy.symbol")
    return str(symbol) if symbol else function.name


def _is_tensor_function(function) -> bool:
    return any(op.dialect in ("tensor", "linalg") for op in function.operations())


def plan_module(module) -> P.ModulePlan:
    """Plan every defined function of `module`, or raise `Unsupported`. The backend passes
    that move reduced middle axes last and give thread-chunked ranges back their range run here
    too (they change nothing the second time), for IR that reaches the translator without the
    backend's passes (a `.ppyir` read directly)."""
    from .passes import reductions_to_trailing_axes, thread_chunks_to_ranges

    reductions_to_trailing_axes(module)
    thread_chunks_to_ranges(module)
    functions = []
    notes: list[str] = []
    bodies = set()
    for function in module.functions.values():
        for op in function.operations():
            if op.dialect == "parallel":
                bodies.add(op.attributes["callee"].name)
    scalar = ScalarEmitter(module)
    for function in module.functions.values():
        if function.is_declaration:
            continue
        if function.name in bodies:
            continue  # a parallel body: emitted as device code by its caller
        symbol = _symbol_of(function)
        if _is_tensor_function(function):
            planned = _TensorTranslator(module, function, symbol).run()
            functions.append(planned)
            kinds = ", ".join(k.kind for k in planned.kernels)
            notes.append(f"@{function.name}: {len(planned.kernels)} kernel(s): {kinds}")
        else:
            planned = scalar.function(function, symbol)
            functions.append(planned)
            if planned.kernels:
                notes.append(f"@{function.name}: {len(planned.kernels)} parallel kernel(s)")
    result = P.ModulePlan(module.name, functions, notes)
    result.device_sources = list(scalar.device_sources)
    result.parallel_kernels = list(scalar.kernels)
    return result
