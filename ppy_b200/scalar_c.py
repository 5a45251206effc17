"""Core-dialect functions as C++: the host side of scalar functions and the device side
of `parallel.*` bodies.

A function becomes one C++ function returning the reference's status
(ppy_runtime/abi.py:25-35) with its result through a pointer, exactly the native ABI
of the reference's LLVM backend (backend/llvm/from_ir.py:1-13): every block is a
label, block arguments are variables assigned before the branch, stack slots
(`core.alloca`) are local arrays, and every guard, Python-semantics overflow and
failed extern goes to `return PPY_STATUS_FALLBACK`. Device copies of the same
functions are emitted for the bodies a `parallel.*` operation runs, and each
`parallel.*` operation becomes a kernel over its range (kernels are described in
`ParallelKernel` and spelled here too).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

from . import plan as P

__all__ = ["ScalarEmitter", "Unsupported", "c_literal"]


class Unsupported(Exception):
    """IR the backend does not take: what, and the capability it lacks."""

    def __init__(self, what: str, capability: str = "") -> None:
        super().__init__(what)
        self.what = what
        self.capability = capability


def c_literal(value, dtype: str) -> str:
    """A C++ literal of `value` as `dtype`, rounded as the reference rounds a constant
    (a Python float to double, then to the element type)."""
    if dtype == "bool":
        return "true" if value else "false"
    if P.is_float(dtype):
        v = float(value)
        if math.isnan(v):
            text = "(double)NAN"
        elif math.isinf(v):
            text = "(double)INFINITY" if v > 0 else "(-(double)INFINITY)"
        else:
            text = repr(v)
            if "e" not in text and "." not in text and "n" not in text:
                text += ".0"
        if dtype == "f64":
            return f"({text})"
        if dtype == "f32":
            return f"((float){text})"
        return f"__float2bfloat16_rn((float){text})"
    v = int(value)
    if dtype in ("i64", "index"):
        if v == -(1 << 63):
            return "((int64_t)(-9223372036854775807LL - 1))"
        return f"((int64_t){v}LL)"
    if dtype.startswith("u"):
        return f"(({P.ctype(dtype)}){v}ULL)"
    return f"(({P.ctype(dtype)}){v})"


#: `ppy_math_unary` / `ppy_math_binary` selectors (src/ppy_runtime/stdlib.c:497-528,
#: table in lowering/stdlib.py:61-64), as device functions.
MATH_UNARY = {0: "asin", 1: "acos", 2: "atan", 3: "sinh", 4: "cosh", 5: "tanh", 6: "asinh",
              7: "acosh", 8: "atanh", 9: "log1p", 10: "expm1", 11: "erf", 12: "erfc",
              13: "cbrt", 14: "exp2", 16: "tan"}
MATH_BINARY = {0: "atan2", 1: "copysign", 2: "fmod"}
#: libm externs a body may call by name, with their arity.
LIBM = {"sqrt": 1, "exp": 1, "log": 1, "sin": 1, "cos": 1, "tan": 1, "fabs": 1, "floor": 1,
        "ceil": 1, "trunc": 1, "pow": 2, "atan2": 2, "fmod": 2, "tanh": 1, "log2": 1,
        "log10": 1, "exp2": 1, "expm1": 1, "log1p": 1, "hypot": 2, "copysign": 2}


@dataclass
class ParallelKernel:
    """One `parallel.for/reduce/map` operation as a kernel over its range."""

    name: str
    kind: str  # "for" | "reduce" | "map"
    body: str  # device function name of the body
    captures: list  # (C type, name)
    result: str | None = None  # reduce: element dtype
    reduce: str | None = None
    reassociate: bool = True
    out_dtype: str | None = None  # map
    extra: dict = field(default_factory=dict)


def _ctype_of(t) -> str:
    text = str(t)
    if text in P.CTYPES:
        return P.ctype(text)
    if text.startswith("ptr<"):
        return _ctype_of(t.pointee) + "*"
    raise Unsupported(f"a value of type {text}", "scalars, pointers and buffers")


def _dtype(t) -> str:
    text = str(t)
    if text not in P.CTYPES:
        raise Unsupported(f"a value of type {text}")
    return text


def _is_buffer(t) -> bool:
    return str(t).startswith("buffer<")


def _is_ptr(t) -> bool:
    return str(t).startswith("ptr<")


class _FunctionEmitter:
    """One IR function as C++ (host or device flavour)."""

    def __init__(self, owner: "ScalarEmitter", function, device: bool,
                 span: tuple[int, int] | None = None) -> None:
        self.owner = owner
        self.function = function
        self.device = device
        # for the body of a parallel.for/reduce: the positions of its (begin, end) params
        self.span = span
        self.names: dict[int, str] = {}
        self.decls: list[str] = []
        self.lines: list[str] = []
        self.counter = 0

    def name(self, value) -> str:
        found = self.names.get(id(value))
        if found is None:
            self.counter += 1
            found = f"v{self.counter}"
            self.names[id(value)] = found
            t = value.type
            if _is_buffer(t):
                element = _ctype_of(t.element)
                self.decls.append(f"{element}* {found}_ptr = nullptr; int64_t {found}_len = 0;")
            elif str(t) in ("void", "()"):
                pass
            else:
                self.decls.append(f"{_ctype_of(t)} {found}{{}};")
        return found

    def signature(self, cname: str) -> str:
        params = []
        for (pname, t), argument in zip(self.function.params, self.function.entry.arguments):
            var = self.name(argument)
            if _is_buffer(t):
                params.append(f"{_ctype_of(t.element)}* {var}_ptr_in")
                params.append(f"int64_t {var}_len_in")
            else:
                params.append(f"{_ctype_of(t)} {var}_in")
        results = list(self.function.results)
        if len(results) > 1:
            raise Unsupported(f"@{self.function.name}: several results")
        if results:
            params.append(f"{_ctype_of(results[0])}* ret")
        recursive = any(
            op.name == "core.call" and op.attributes["callee"].name == self.function.name
            for op in self.function.operations()
        )
        inline = "__noinline__" if recursive else "__forceinline__"
        qualifier = f"static __device__ {inline}" if self.device else "static"
        return f"{qualifier} int32_t {cname}({', '.join(params) or 'void'})"

    def emit(self, cname: str) -> str:
        fn = self.function
        head = self.signature(cname)
        # Parameters arrive under *_in names and are copied into their variables so a
        # block may reassign nothing it should not.
        entry_copies = []
        for (pname, t), argument in zip(fn.params, fn.entry.arguments):
            var = self.names[id(argument)]
            if _is_buffer(t):
                entry_copies.append(f"{var}_ptr = {var}_ptr_in; {var}_len = {var}_len_in;")
            else:
                entry_copies.append(f"{var} = {var}_in;")
        blocks = list(fn.body.blocks)
        self.labels = {id(b): f"bb{i}" for i, b in enumerate(blocks)}
        for block in blocks:
            for argument in block.arguments:
                if block is not blocks[0]:
                    self.name(argument)
        # Device code bounds every loop: a header reached more than PPYB200_LOOP_LIMIT
        # times in one call returns PPY_STATUS_RAISED instead of spinning forever (a
        # body such as Collatz never ends for a start <= 0, on the CPU as here). A
        # parallel body called on a run of indices [begin, end) gets the bound times the
        # run's length: the same allowance per index.
        index = {id(b): i for i, b in enumerate(blocks)}
        headers = set()
        if self.device:
            for i, block in enumerate(blocks):
                terminator = block.operations[-1] if block.operations else None
                for successor in getattr(terminator, "successors", []) or []:
                    if index[id(successor.block)] <= i:
                        headers.add(id(successor.block))
        body: list[str] = []
        for block in blocks:
            body.append(f"{self.labels[id(block)]}:;")
            if id(block) in headers:
                body.append("  if (++loop_trips > trip_limit) return PPY_STATUS_RAISED;")
            for op in block.operations:
                body.extend("  " + line for line in self.op(op))
        text = [head + " {"]
        if headers:
            text.append("  uint64_t loop_trips = 0;")
            if self.span is not None:
                params = [f"{self.names[id(a)]}_in" for a in fn.entry.arguments]
                b, e = (params[i] for i in self.span)
                text.append(f"  const uint64_t trip_limit = (uint64_t)PPYB200_LOOP_LIMIT * "
                            f"(uint64_t)({e} > {b} ? {e} - {b} : 1);")
            else:
                text.append("  const uint64_t trip_limit = PPYB200_LOOP_LIMIT;")
        text += ["  " + d for d in self.decls]
        text += ["  " + c for c in entry_copies]
        text += [f"  goto {self.labels[id(blocks[0])]};"]
        text += body
        text += ["}"]
        return "\n".join(text)

    # ---------------------------------------------------------------- helpers

    def v(self, value) -> str:
        return self.name(value)

    def fallback(self) -> str:
        return "return PPY_STATUS_FALLBACK;"

    def branch(self, successor) -> list[str]:
        target = successor.block
        lines = []
        arguments = list(successor.arguments)
        params = list(target.arguments)
        if arguments:
            temps = []
            for i, (param, arg) in enumerate(zip(params, arguments)):
                ct = _ctype_of(param.type)
                temps.append(f"{ct} p{i} = {self.v(arg)};")
            assigns = [f"{self.v(param)} = p{i};" for i, param in enumerate(params)]
            lines.append("{ " + " ".join(temps + assigns) + " }")
        lines.append(f"goto {self.labels[id(target)]};")
        return lines

    # ---------------------------------------------------------------- operations

    def op(self, op) -> list[str]:  # noqa: C901 - one case per operation
        name = op.name
        dialect, local = name.split(".", 1)
        if dialect == "parallel":
            if self.device:
                raise Unsupported("a parallel loop inside a parallel body",
                                  "parallel loops at the top level of a function")
            return self.owner.parallel(self, op)
        if dialect == "math":
            r = self.v(op.results[0])
            args = ", ".join(self.v(a) for a in op.operands)
            fn = "fabs" if local == "abs" else local
            return [f"{r} = {fn}({args});"]
        if dialect == "special":
            r = self.v(op.results[0])
            fn = {"gamma": "tgamma", "gammaln": "lgamma", "bessel_j0": "j0", "bessel_j1": "j1",
                  "bessel_y0": "y0", "bessel_y1": "y1"}.get(local, local)
            if fn in ("ndtr", "logit"):
                fn = "ppyb200::" + fn
            return [f"{r} = {fn}({self.v(op.operands[0])});"]
        if dialect == "concurrency":
            # parallel.range already split into host-thread chunks (LowerParallel's threads
            # route, lower_parallel.py:141-318): the GPU wants the whole range
            raise Unsupported(f"{name}: ppy.parallel.range lowered to host threads",
                              "parallel.reduce/for/map as the IR op: set `[tool.ppy.parallel] "
                              "backend = \"openmp\"` in pyproject.toml")
        if dialect != "core":
            raise Unsupported(f"{name}", "core, math, special and parallel operations")
        a = op.attributes
        if local == "const":
            r = self.v(op.results[0])
            t = op.results[0].type
            if _is_ptr(t):
                return [f"{r} = nullptr;"]
            return [f"{r} = {c_literal(a['value'], _dtype(t))};"]
        if local in ("add", "sub", "mul"):
            return self.arith(op, local)
        if local in ("div", "mod"):
            return self.divmod(op, local)
        if local == "neg":
            r, x = self.v(op.results[0]), self.v(op.operands[0])
            t = _dtype(op.results[0].type)
            if P.is_float(t) or a.get("overflow", "python") in ("wrap", "native", "proven"):
                return [f"{r} = ({P.ctype(t)})(0 - {x});" if not P.is_float(t) else f"{r} = -{x};"]
            return [f"if (ppyb200::sub_overflows(0, {x}, &{r})) {self.fallback()}"]
        if local in ("and", "or", "xor"):
            sym = {"and": "&", "or": "|", "xor": "^"}[local]
            r = self.v(op.results[0])
            return [f"{r} = {self.v(op.operands[0])} {sym} {self.v(op.operands[1])};"]
        if local in ("shl", "shr"):
            r = self.v(op.results[0])
            x, s = self.v(op.operands[0]), self.v(op.operands[1])
            if local == "shr":
                return [f"{r} = {x} >> {s};"]
            lines = [f"{r} = ({P.ctype(_dtype(op.results[0].type))})((uint64_t){x} << {s});"]
            if a.get("overflow", "wrap") not in ("wrap", "native"):
                lines.append(f"if (({r} >> {s}) != {x}) {self.fallback()}")
            return lines
        if local == "cmp":
            sym = {"eq": "==", "ne": "!=", "lt": "<", "le": "<=", "gt": ">", "ge": ">="}[
                str(a["predicate"])]
            return [f"{self.v(op.results[0])} = ({self.v(op.operands[0])} {sym} "
                    f"{self.v(op.operands[1])});"]
        if local == "select":
            c, x, y = (self.v(v) for v in op.operands)
            return [f"{self.v(op.results[0])} = {c} ? {x} : {y};"]
        if local == "cast":
            r = self.v(op.results[0])
            return [f"{r} = ({_ctype_of(op.results[0].type)}){self.v(op.operands[0])};"]
        if local == "br":
            return self.branch(op.successors[0])
        if local == "cond_br":
            then = self.branch(op.successors[0])
            other = self.branch(op.successors[1])
            return [f"if ({self.v(op.operands[0])}) {{"] + ["  " + t for t in then] + [
                "} else {"] + ["  " + o for o in other] + ["}"]
        if local == "ret":
            if op.operands:
                return [f"*ret = {self.v(op.operands[0])};", "return PPY_STATUS_OK;"]
            return ["return PPY_STATUS_OK;"]
        if local == "unreachable":
            return ["return PPY_STATUS_RAISED;"]
        if local == "alloca":
            r = self.v(op.results[0])
            count = int(a.get("count", 1) or 1)
            element = _ctype_of(op.results[0].type.pointee)
            self.counter += 1
            slot = f"slot{self.counter}"
            self.decls.append(f"{element} {slot}[{count}];")
            return [f"{r} = {slot};"]
        if local == "load":
            return [f"{self.v(op.results[0])} = *{self.v(op.operands[0])};"]
        if local == "store":
            return [f"*{self.v(op.operands[1])} = {self.v(op.operands[0])};"]
        if local == "ptr_offset":
            return [f"{self.v(op.results[0])} = {self.v(op.operands[0])} + "
                    f"{self.v(op.operands[1])};"]
        if local == "buffer_data":
            return [f"{self.v(op.results[0])} = {self.v(op.operands[0])}_ptr;"]
        if local == "buffer_len":
            return [f"{self.v(op.results[0])} = {self.v(op.operands[0])}_len;"]
        if local == "buffer_load":
            b, i = self.v(op.operands[0]), self.v(op.operands[1])
            return [f"{self.v(op.results[0])} = {b}_ptr[{i}];"]
        if local == "buffer_store":
            x, b, i = (self.v(v) for v in op.operands)
            return [f"{b}_ptr[{i}] = {x};"]
        if local == "guard":
            return [f"if (!({self.v(op.operands[0])})) {self.fallback()}"]
        if local == "call":
            return self.call(op)
        if local == "call_extern":
            return self.extern(op)
        raise Unsupported(f"{name}", "the core operations of scalar code")

    def arith(self, op, local: str) -> list[str]:
        r = self.v(op.results[0])
        x, y = self.v(op.operands[0]), self.v(op.operands[1])
        t = _dtype(op.results[0].type)
        sym = {"add": "+", "sub": "-", "mul": "*"}[local]
        if P.is_float(t):
            return [f"{r} = {x} {sym} {y};"]
        overflow = op.attributes.get("overflow", "python")
        ct = P.ctype(t)
        if overflow in ("wrap", "native", "proven") or t not in ("i64", "index"):
            unsigned = "uint64_t" if P.size_of(t) == 8 else "uint32_t"
            return [f"{r} = ({ct})(({unsigned}){x} {sym} ({unsigned}){y});"]
        return [f"if (ppyb200::{local}_overflows({x}, {y}, &{r})) {self.fallback()}"]

    def divmod(self, op, local: str) -> list[str]:
        r = self.v(op.results[0])
        x, y = self.v(op.operands[0]), self.v(op.operands[1])
        t = _dtype(op.results[0].type)
        if P.is_float(t):
            if local == "mod":
                raise Unsupported("a float remainder", "Python's float %")
            return [f"{r} = {x} / {y};"]
        lines = []
        if op.attributes.get("overflow", "python") not in ("wrap", "native") and t in ("i64",
                                                                                       "index"):
            lines.append(f"if ({x} == (int64_t)(-9223372036854775807LL - 1) && {y} == -1) "
                         f"{self.fallback()}")
        rounding = op.attributes.get("rounding", "floor")
        if rounding == "trunc" or t.startswith("u"):
            lines.append(f"{r} = {x} {'/' if local == 'div' else '%'} {y};")
            return lines
        power = self._power_of_two(op.operands[1])
        if power is not None:
            if local == "div":
                lines.append(f"{r} = {x} >> {power};")
            else:
                lines.append(f"{r} = {x} & {(1 << power) - 1};")
            return lines
        fn = "floordiv" if local == "div" else "floormod"
        lines.append(f"{r} = ppyb200::{fn}((int64_t){x}, (int64_t){y});")
        return lines

    @staticmethod
    def _power_of_two(value):
        owner = value.owner
        if getattr(owner, "name", None) != "core.const":
            return None
        v = owner.attributes.get("value")
        if isinstance(v, bool) or not isinstance(v, int) or v <= 0 or v & (v - 1):
            return None
        return v.bit_length() - 1

    def call(self, op) -> list[str]:
        callee = op.attributes["callee"].name
        target = self.owner.module.functions.get(callee)
        if target is None or target.is_declaration:
            raise Unsupported(f"a call to @{callee}", "calls to functions of the module")
        cname = self.owner.device_function(target) if self.device else self.owner.host_name(target)
        args = []
        for value in op.operands:
            if _is_buffer(value.type):
                args += [f"{self.v(value)}_ptr", f"{self.v(value)}_len"]
            else:
                args.append(self.v(value))
        lines = []
        if op.results:
            args.append(f"&{self.v(op.results[0])}")
        lines.append(f"{{ int32_t s = {cname}({', '.join(args)}); if (s != PPY_STATUS_OK) "
                     f"return s; }}")
        return lines

    def extern(self, op) -> list[str]:
        callee = str(op.attributes["callee"].name if hasattr(op.attributes["callee"], "name")
                     else op.attributes["callee"])
        args = [self.v(v) for v in op.operands]
        r = self.v(op.results[0]) if op.results else None
        if callee == "ppy_math_unary":
            selector = self._const(op.operands[0])
            fn = MATH_UNARY.get(selector, "fabs")
            return [f"{r} = {fn}({args[1]});"]
        if callee == "ppy_math_binary":
            selector = self._const(op.operands[0])
            fn = MATH_BINARY.get(selector, "fmod")
            return [f"{r} = {fn}({args[1]}, {args[2]});"]
        if callee in LIBM and LIBM[callee] == len(args) and r is not None:
            return [f"{r} = {callee}({', '.join(args)});"]
        raise Unsupported(f"a call to the extern {callee}", "math externs")

    @staticmethod
    def _const(value) -> int:
        owner = value.owner
        if getattr(owner, "name", None) != "core.const":
            raise Unsupported("a math extern with a computed selector")
        return int(owner.attributes["value"])


class ScalarEmitter:
    """Emits scalar functions, their parallel kernels, and the device copies they need."""

    def __init__(self, module) -> None:
        self.module = module
        self.device_done: dict[str, str] = {}
        self.device_sources: list[str] = []
        self.kernels: list[ParallelKernel] = []

    @staticmethod
    def host_name(function) -> str:
        return f"host_{function.name}"

    def device_function(self, function, span: tuple[int, int] | None = None) -> str:
        cname = f"dev_{function.name}"
        if function.name in self.device_done:
            return cname
        self.device_done[function.name] = cname
        text = _FunctionEmitter(self, function, device=True, span=span).emit(cname)
        self.device_sources.append(text)
        return cname

    def parallel(self, emitter: _FunctionEmitter, op) -> list[str]:
        callee = self.module.functions[op.attributes["callee"].name]
        kind = op.local_name if hasattr(op, "local_name") else op.name.split(".", 1)[1]
        # for and reduce bodies loop over their own [begin, end): the kernel hands them runs
        # of indices; a map body takes one index
        n = len(callee.params)
        span = {"for": (n - 2, n - 1), "reduce": (n - 3, n - 2)}.get(kind)
        body = self.device_function(callee, span)
        operands = list(op.operands)
        trailing = {"for": 2, "reduce": 3, "map": 3}[kind]
        captures = operands[: len(operands) - trailing]
        capture_decls = []
        for i, value in enumerate(captures):
            if _is_buffer(value.type):
                capture_decls.append((f"{_ctype_of(value.type.element)}*", f"c{i}_ptr"))
                capture_decls.append(("int64_t", f"c{i}_len"))
            else:
                capture_decls.append((_ctype_of(value.type), f"c{i}"))
        name = f"par_{emitter.function.name}_{len(self.kernels)}"
        kernel = ParallelKernel(name, kind, body, capture_decls)
        if kind == "reduce":
            kernel.result = _dtype(op.results[0].type)
            kernel.reduce = str(op.attributes["op"])
            kernel.reassociate = bool(op.attributes.get("reassociate", True))
            if P.is_float(kernel.result) and not kernel.reassociate:
                raise Unsupported("a floating-point parallel reduction that may not reassociate",
                                  "integer reductions, or float ones marked reassociate")
        if kind == "map":
            kernel.out_dtype = _dtype(op.operands[-1].type.pointee)
        self.kernels.append(kernel)
        args = []
        for value in captures:
            if _is_buffer(value.type):
                args += [f"{emitter.v(value)}_ptr", f"{emitter.v(value)}_len"]
            else:
                args.append(emitter.v(value))
        begin, end = operands[len(captures)], operands[len(captures) + 1]
        args += [emitter.v(begin), emitter.v(end)]
        if kind == "reduce":
            args.append(emitter.v(operands[-1]))
            args.append(f"&{emitter.v(op.results[0])}")
        if kind == "map":
            args.append(emitter.v(operands[-1]))
        return [f"{{ int32_t s = launch_{name}({', '.join(args)}); if (s != PPY_STATUS_OK) "
                f"return s; }}"]

    def function(self, function, symbol: str) -> P.ScalarFunction:
        before = len(self.kernels)
        source = _FunctionEmitter(self, function, device=False).emit(self.host_name(function))
        params = []
        for pname, t in function.params:
            if _is_buffer(t):
                params.append(P.Param(pname, "buffer", _dtype(t.element), role="inout"))
            elif _is_ptr(t):
                params.append(P.Param(pname, "ptr", _dtype(t.pointee)))
            else:
                params.append(P.Param(pname, "scalar", _dtype(t)))
        results = list(function.results)
        result = _dtype(results[0]) if results else None
        return P.ScalarFunction(function.name, symbol, params, result, source,
                                [], self.kernels[before:])
