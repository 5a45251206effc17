"""Backend-stage passes of the b200 backend.

`CommonTensorsToBuffers` makes functions written over `ppy.Tensor` parameters (PPy source
typed by the `b200_tensor` plugin, `ppy_b200.tensor_plugin`) look like the tensor functions of
a `.ppyir` module, which take buffers and `tensor.load` / `tensor.store` them
(lower_tensor.py:125-131 of the reference: a tensor crosses a call as a buffer):

    %a: tensor<f32, N>  (a parameter)  ->  %a: buffer<f32>, %x = tensor.load %a
    b200.assign %out, %v               ->  tensor.store %v, %out      (%out: buffer<f32>)
    b200.fill %s {dtype}               ->  tensor.fill %s'            (%s' the constant in dtype)

and first forwards the stack slots the frontend gives every local tensor variable
(`core.alloca` of a tensor, `core.store`, `core.load` in one block) to the values stored, so
that the tensor operations read one another directly.

The backend's C ABI then passes every such parameter as a pointer and a length, like any
buffer, and `role` in the manifest says whether the call reads it, writes it or both.
"""

from __future__ import annotations

from ppy_compiler.ir import BufferType, Builder, PtrType, Successor
from ppy_compiler.ir.dialects import core
from ppy_compiler.ir.dialects import tensor as tensor_dialect
from ppy_compiler.ir.passes import Pass, PassContext

from .scalar_c import Unsupported

__all__ = ["CommonTensorsToBuffers", "common_tensors_to_buffers", "ReductionsToTrailingAxes",
           "reductions_to_trailing_axes", "ThreadChunksToRanges", "thread_chunks_to_ranges"]


def _cast(value, dtype: str):
    """A constant's value as the element type `dtype` takes it."""
    if dtype.startswith(("i", "u")):
        return int(value)
    return float(value)


def common_tensors_to_buffers(module) -> bool:
    """Rewrite `module` in place; True if anything changed."""
    changed = False
    for function in module.functions.values():
        if function.is_declaration:
            continue
        changed |= _slots(function)
        changed |= _fills(function)
        changed |= _parameters(function)
    return changed


def _slots(function) -> bool:
    """Forward `core.store` to `core.load` through tensor stack slots of a one-block function."""
    blocks = function.body.blocks
    if len(blocks) != 1:
        return False
    slots = set()
    current: dict[int, object] = {}
    dead = []
    changed = False
    for op in list(blocks[0].operations):
        if op.name == "core.alloca":
            t = op.results[0].type
            if isinstance(t, PtrType) and tensor_dialect.describe(t.pointee) is not None:
                slots.add(id(op.results[0]))
                dead.append(op)
        elif op.name == "core.store" and id(op.operands[1]) in slots:
            current[id(op.operands[1])] = op.operands[0]
            op.erase()
            changed = True
        elif op.name == "core.load" and id(op.operands[0]) in slots:
            value = current.get(id(op.operands[0]))
            if value is None:
                raise Unsupported(f"@{function.name}: a tensor variable read before it is set")
            op.results[0].replace_all_uses_with(value)
            op.erase()
            changed = True
    for op in dead:
        if not op.results[0].uses:
            op.erase()
    return changed


def _fills(function) -> bool:
    changed = False
    for op in list(function.operations()):
        if op.name != "b200.fill":
            continue
        scalar = op.operands[0]
        result = op.results[0]
        dtype = tensor_dialect.describe(result.type).dtype
        b = Builder().before(op)
        owner = scalar.owner
        if getattr(owner, "name", None) == "core.const":
            scalar = core.const(b, _cast(owner.attributes["value"], str(dtype)), dtype)
        elif scalar.type != dtype:
            raise Unsupported(f"@{function.name}: bt.full of a {scalar.type} value as {dtype}",
                              "bt.full of a constant, or of a scalar of the element type")
        fill = b.create("tensor.fill", (scalar,), (result.type,))
        result.replace_all_uses_with(fill.results[0])
        op.erase()
        changed = True
    return changed


def _parameters(function) -> bool:
    entry = function.entry
    if entry is None:
        return False
    if any(tensor_dialect.describe(t) is not None for t in function.results):
        raise Unsupported(f"@{function.name}: a tensor result",
                          "results written into ppy.Mut[ppy.Tensor] parameters with bt.assign")
    params = list(function.params)
    changed = False
    for index, (name, declared) in enumerate(function.params):
        info = tensor_dialect.describe(declared)
        if info is None:
            continue
        argument = entry.arguments[index]
        buffer = BufferType(info.dtype)
        argument.type = buffer
        params[index] = (name, buffer)
        # writes: b200.assign %arg, %v  ->  tensor.store %v, %arg (the value broadcast first)
        for user, slot in list(argument.uses):
            if getattr(user, "name", None) == "b200.assign" and slot == 0:
                value = user.operands[1]
                b = Builder().before(user)
                if tuple(tensor_dialect.describe(value.type).shape) != tuple(info.shape):
                    value = b.create("tensor.broadcast", (value,), (declared,)).results[0]
                b.create("tensor.store", (value, argument), ())
                user.erase()
        # reads: one load at the top of the function (the stores just made keep the buffer)
        reads = [(user, slot) for user, slot in argument.uses
                 if not (getattr(user, "name", None) == "tensor.store" and slot == 1)]
        if reads:
            first = entry.operations[0] if entry.operations else None
            b = Builder(entry) if first is None else Builder().before(first)
            load = b.create("tensor.load", (argument,), (declared,), result_names=(name,))
            loaded = load.results[0]
            for user, slot in reads:
                user.set_operand(slot, loaded)
        changed = True
    if changed:
        function.params = tuple(params)
        for attributes in function.param_attributes:
            attributes.pop("ppy.kind", None)
    return changed


class CommonTensorsToBuffers(Pass):
    """Backend-stage pass: tensor parameters become buffers (see the module docstring)."""

    name = "b200-common-tensors-to-buffers"

    def run(self, module, ctx: PassContext) -> bool:
        changed = common_tensors_to_buffers(module)
        if changed:
            ctx.invalidate()
        return changed


def reductions_to_trailing_axes(module) -> bool:
    """Rewrite `linalg.dot` as a product and a reduction, and every `tensor.reduce` over axes that are neither all of its input's axes nor a
    leading or trailing run of them into a transpose that moves them last (the kept axes
    first, both in order) and a reduce over the trailing axes; with keepdims a reshape gives
    back the unit-axis shape, which has the same layout. Each output element then folds its
    elements in the row-major order of the reduced axes, as the reference's row-major loop
    does (lower_tensor.py:733-754). True if anything changed."""
    changed = False
    for function in module.functions.values():
        if function.is_declaration:
            continue
        for op in list(function.operations()):
            if op.name == "linalg.dot":
                # sum of a[k] * b[k] from zero (lower_tensor.py:792-802): an elementwise
                # product and a whole-vector add reduction
                b = Builder().before(op)
                product = tensor_dialect.elementwise(b, "mul", op.operands[0], op.operands[1])
                total = tensor_dialect.reduce(b, product, (0,), "add", keepdims=False)
                op.results[0].replace_all_uses_with(total)
                op.erase()
                changed = True
                continue
            if op.name != "tensor.reduce":
                continue
            source = op.operands[0]
            rank = len(tensor_dialect.describe(source.type).shape)
            axes = tuple(sorted(int(a) for a in op.attributes["axes"]))
            if (not axes or axes == tuple(range(rank)) or axes == tuple(range(len(axes)))
                    or axes == tuple(range(rank - len(axes), rank))):
                continue
            kept = [d for d in range(rank) if d not in axes]
            b = Builder().before(op)
            moved = tensor_dialect.transpose(b, source, tuple(kept) + axes)
            result = tensor_dialect.reduce(b, moved, tuple(range(len(kept), rank)),
                                           str(op.attributes["op"]), keepdims=False)
            if bool(op.attributes.get("keepdims", False)):
                result = tensor_dialect.reshape(b, result,
                                                tensor_dialect.describe(op.results[0].type).shape)
            op.results[0].replace_all_uses_with(result)
            op.erase()
            changed = True
    return changed


class ReductionsToTrailingAxes(Pass):
    """Backend-stage pass: `linalg.dot` becomes a product and a reduction, reductions over
    middle axes a transpose and a reduction over trailing axes (see
    `reductions_to_trailing_axes`)."""

    name = "b200-reductions-to-trailing-axes"

    def run(self, module, ctx: PassContext) -> bool:
        changed = reductions_to_trailing_axes(module)
        if changed:
            ctx.invalidate()
        return changed


# ---------------------------------------------------------------- thread chunks back into ranges


def _is_float(t) -> bool:
    return str(t).startswith(("f", "bf"))


def _drop_unreachable(function) -> None:
    blocks = function.body.blocks
    reached, todo = set(), [blocks[0]]
    while todo:
        block = todo.pop()
        if id(block) in reached:
            continue
        reached.add(id(block))
        todo.extend(block.successors)
    for block in [b for b in blocks if id(b) not in reached]:
        for op in reversed(list(block.operations)):
            op.erase()
        blocks.remove(block)


def thread_chunks_to_ranges(module) -> bool:
    """Give a `parallel.range` loop that PPy's default `threads` route split into host-thread
    chunks back its range. That route (lower_parallel.py:141-318) leaves, per loop, a branch on
    the range's size between a serial block -- one call of the chunk body `@f__parN` over the
    whole range, the initial accumulator last -- and a spawn block that calls it on eight
    chunks with `concurrency.spawn` and folds their partials in order. The serial call has
    the operands, in the order, of the `parallel.reduce` / `parallel.for` that the `openmp`
    route keeps (parallel.py:562-610): it becomes that op (for a reduction, its kind from how
    the spawn block combines the initial value, reassociating integers only, as the frontend
    decides at ast_to_ir.py:4026), the branch goes to the serial block, and the spawn block
    and the task wrappers nothing calls any more go. True if anything changed."""
    changed = False
    for function in list(module.functions.values()):
        if function.is_declaration:
            continue
        for block in list(function.body.blocks):
            if not block.operations:
                continue
            branch = block.operations[-1]
            if branch.name != "core.cond_br" or len(branch.successors) != 2:
                continue
            serial, spawn = branch.successors[0].block, branch.successors[1].block
            if not (serial.name.startswith("par.serial") and spawn.name.startswith("par.spawn")):
                continue
            calls = [op for op in serial.operations if op.name == "core.call"]
            if len(calls) != 1 or not any(op.name == "concurrency.spawn"
                                          for op in spawn.operations):
                continue
            call = calls[0]
            body = module.functions.get(call.attributes["callee"].name)
            if body is None or body.attributes.get("ppy.synthesized") != "parallel":
                continue
            b = Builder().before(call)
            if call.results:
                init = call.operands[-1]
                combine = next((op.name for op in spawn.operations
                                if op.name in ("core.add", "core.mul")
                                and any(v is init for v in op.operands)), None)
                if combine is None:
                    continue
                result = call.results[0]
                reduce_op = b.create("parallel.reduce", tuple(call.operands), (result.type,),
                                     {"callee": call.attributes["callee"],
                                      "op": "add" if combine == "core.add" else "mul",
                                      "reassociate": not _is_float(result.type)})
                result.replace_all_uses_with(reduce_op.results[0])
            else:
                b.create("parallel.for", tuple(call.operands), (),
                         {"callee": call.attributes["callee"]})
            call.erase()
            Builder().before(branch).create("core.br", (), (), successors=(Successor(serial),))
            branch.erase()
            _drop_unreachable(function)
            changed = True
    if changed:
        called = {op.attributes["callee"].name for fn in module.functions.values()
                  if not fn.is_declaration for op in fn.operations()
                  if "callee" in op.attributes}
        for name, fn in list(module.functions.items()):
            if fn.attributes.get("ppy.synthesized") == "parallel.reduce" and name not in called:
                del module.functions[name]
    return changed


class ThreadChunksToRanges(Pass):
    """Backend-stage pass: `parallel.range` loops split into host-thread chunks by PPy's default
    `threads` route become whole `parallel.*` ops again (see `thread_chunks_to_ranges`)."""

    name = "b200-thread-chunks-to-ranges"

    def run(self, module, ctx: PassContext) -> bool:
        changed = thread_chunks_to_ranges(module)
        if changed:
            ctx.invalidate()
        return changed
