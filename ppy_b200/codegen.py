"""Kernel plan -> CUDA C++ for sm_100a.

Every kernel is spelled for its plan: the element program is inlined into a
hand-shaped skeleton (vectorized streaming loads, rows held in registers with
warp-shuffle reductions, two-pass reductions over scratch partials), so a fused
group touches HBM once per input byte and once per output byte. Host wrappers give
each IR function the reference's native ABI twice over: `<symbol>` for host memory
(copies in, launches, copies out) and `<symbol>__device` for device memory.
"""

from __future__ import annotations

from . import plan as P
from .scalar_c import ParallelKernel, c_literal

__all__ = ["module_source"]

THREADS = 256
#: Vectors each thread of a map kernel keeps in flight per loop trip.
MAP_UNROLL = 1
#: Resident 256-thread blocks per SM a vectorized map kernel is compiled for (full occupancy).
MAP_MIN_BLOCKS = 0
#: Resident blocks per SM a row kernel is compiled for (0: let the compiler choose).
ROW_MIN_BLOCKS = 0
#: Shared memory a pipelined row kernel may take per block (two row buffers per warp).
ROW_SMEM_LIMIT = 100 * 1024
ROW_STAGES = 3  # rows a warp has in flight: the one it computes and ROW_STAGES - 1 prefetched
#: Threads of a row kernel block when a row takes at most one warp.
ROW_THREADS = 256

_MATH32 = {"sqrt": "sqrtf", "sin": "sinf", "cos": "cosf", "tan": "tanf", "exp": "expf",
           "exp2": "exp2f", "log": "logf", "log2": "log2f", "log10": "log10f",
           "floor": "floorf", "ceil": "ceilf", "trunc": "truncf", "abs": "fabsf"}
_MATH64 = {"abs": "fabs"}
_SPECIAL32 = {"erf": "erff", "erfc": "erfcf", "gamma": "tgammaf", "gammaln": "lgammaf",
              "bessel_j0": "j0f", "bessel_j1": "j1f", "bessel_y0": "y0f", "bessel_y1": "y1f",
              "ndtr": "ppyb200::ndtr", "logit": "ppyb200::logit"}
_SPECIAL64 = {"erf": "erf", "erfc": "erfc", "gamma": "tgamma", "gammaln": "lgamma",
              "bessel_j0": "j0", "bessel_j1": "j1", "bessel_y0": "y0", "bessel_y1": "y1",
              "ndtr": "ppyb200::ndtr", "logit": "ppyb200::logit"}
_CMP = {"eq": "==", "ne": "!=", "lt": "<", "le": "<=", "gt": ">", "ge": ">="}
_COMBINE = {"add": "ppyb200::CombAdd", "mul": "ppyb200::CombMul", "max": "ppyb200::OpMax",
            "min": "ppyb200::OpMin"}


def identity_literal(kind: str, dtype: str) -> str:
    """The fold's starting value (lower_tensor.py:1841-1853)."""
    if kind == "add":
        return c_literal(0.0 if P.is_float(dtype) else 0, dtype)
    if kind == "mul":
        return c_literal(1.0 if P.is_float(dtype) else 1, dtype)
    if P.is_float(dtype):
        return c_literal(float("inf") if kind == "min" else float("-inf"), dtype)
    width = P.size_of(dtype) * 8
    signed = not dtype.startswith("u")
    if kind == "min":
        return c_literal((1 << (width - 1)) - 1 if signed else (1 << width) - 1, dtype)
    return c_literal(-(1 << (width - 1)) if signed else 0, dtype)


def combine_expr(kind: str, acc: str, value: str) -> str:
    return f"{_COMBINE[kind]}::apply({acc}, {value})"


# -- element programs ---------------------------------------------------------------------


def _compute_dtype(dtype: str) -> str:
    """bf16 values are computed in f32 and rounded when stored."""
    return "f32" if dtype == "bf16" else dtype


def stmt_expr(stmt: P.Stmt, arg, dtypes: dict, status: bool = True) -> tuple[str, list[str]]:
    """(expression, prelude lines) of one statement; `arg(name)` spells an argument."""
    op = stmt.op
    t = _compute_dtype(stmt.dtype)
    ct = P.ctype(t)
    a = [arg(x) for x in stmt.args] if op not in ("input",) else []
    if op == "const":
        return c_literal(stmt.attrs["value"], t), []
    if op == "param":
        return f"p_{stmt.attrs['name']}", []
    if op in ("add", "sub", "mul"):
        sym = {"add": "+", "sub": "-", "mul": "*"}[op]
        if P.is_float(t):
            return f"({a[0]} {sym} {a[1]})", []
        overflow = stmt.attrs.get("overflow", "python")
        if overflow in ("wrap", "native", "proven") or t not in ("i64", "index"):
            u = "uint64_t" if P.size_of(t) == 8 else "uint32_t"
            return f"(({ct})(({u}){a[0]} {sym} ({u}){a[1]}))", []
        tmp = f"{stmt.var}_c"
        return tmp, [f"int64_t {tmp}; if (ppyb200::{op}_overflows({a[0]}, {a[1]}, &{tmp})) "
                     f"ppyb200::raise_fallback(status);"]
    if op == "div":
        if P.is_float(t):
            return f"({a[0]} / {a[1]})", []
        return f"ppyb200::floordiv({a[0]}, {a[1]})", []
    if op == "mod":
        return f"ppyb200::floormod({a[0]}, {a[1]})", []
    if op == "neg":
        if P.is_float(t):
            return f"(-{a[0]})", []
        return f"(({ct})(0 - (uint64_t){a[0]}))", []
    if op in ("and", "or", "xor"):
        return f"({a[0]} {dict(zip(('and', 'or', 'xor'), '&|^'))[op]} {a[1]})", []
    if op == "shl":
        return f"(({ct})((uint64_t){a[0]} << {a[1]}))", []
    if op == "shr":
        return f"({a[0]} >> {a[1]})", []
    if op == "cmp":
        return f"({a[0]} {_CMP[stmt.attrs['predicate']]} {a[1]})", []
    if op == "select":
        return f"({a[0]} ? {a[1]} : {a[2]})", []
    if op == "cast":
        source = _compute_dtype(dtypes[stmt.args[0]])
        if source == t:
            return a[0], []
        return f"ppyb200::convert<{ct}, {P.ctype(source)}>({a[0]})", []
    if op == "math":
        fn = stmt.attrs["fn"]
        name = _MATH32.get(fn, fn + "f") if t == "f32" else _MATH64.get(fn, fn)
        return f"{name}({a[0]})", []
    if op == "pow":
        return f"{'powf' if t == 'f32' else 'pow'}({a[0]}, {a[1]})", []
    if op == "special":
        fn = stmt.attrs["fn"]
        name = (_SPECIAL32 if t == "f32" else _SPECIAL64)[fn]
        return f"{name}({a[0]})", []
    raise ValueError(f"statement {op} has no device spelling")


def needs_status(program: list) -> bool:
    for s in program:
        if s.op in ("add", "sub", "mul") and not P.is_float(s.dtype) and s.dtype in (
            "i64", "index"
        ) and s.attrs.get("overflow", "python") == "python":
            return True
    return False


# -- access classes ---------------------------------------------------------------------


def presence(shape: tuple, frame: tuple) -> tuple:
    """Per frame dim: does `shape` (right-aligned, NumPy broadcasting) vary there?"""
    padded = (1,) * (len(frame) - len(shape)) + tuple(shape)
    out = []
    for s, f in zip(padded, frame):
        if s == f and f != 1:
            out.append(True)
        elif s == 1:
            out.append(False)
        else:
            raise ValueError(f"{shape} does not broadcast to {frame}")
    return tuple(out)


def coalesce(frame: tuple, flags: list) -> tuple[list, list]:
    """Drop unit dims and merge neighbours every operand treats alike.
    Returns (dims, per-operand presence) where dims are lists of frame dims."""
    keep = [i for i, d in enumerate(frame) if d != 1]
    dims: list[list] = []
    pres: list[list] = [[] for _ in flags]
    for i in keep:
        if dims and all(f[i] == p[-1] for f, p in zip(flags, pres)):
            dims[-1].append(frame[i])
            continue
        dims.append([frame[i]])
        for f, p in zip(flags, pres):
            p.append(f[i])
    return dims, pres


def dim_expr(parts: list) -> str:
    return " * ".join(P.spell_dims(tuple(parts))) if parts else "(int64_t)1"


# -- kernels ------------------------------------------------------------------------------


class _Source:
    def __init__(self) -> None:
        self.kernels: list[str] = []
        self.host: list[str] = []
        self.exports: list[str] = []


def _kernel_params(kernel, extra: list[str]) -> list[str]:
    params = []
    for i, operand in enumerate(kernel.inputs):
        params.append(f"const {P.ctype(operand.dtype)}* __restrict__ in{i}")
    for i, out in enumerate(getattr(kernel, "outputs", [])):
        params.append(f"{P.ctype(out.operand.dtype)}* __restrict__ out{i}")
    return params + extra


def _scalar_params(program: list, params_by_name: dict) -> list[tuple[str, str]]:
    seen = []
    for s in program:
        if s.op == "param" and s.attrs["name"] not in [n for n, _ in seen]:
            seen.append((s.attrs["name"], params_by_name[s.attrs["name"]].dtype))
    return seen


def _program_lines(program: list, value_of, dtypes: dict, indent: str,
                   skip=lambda s: False) -> list[str]:
    """Straight-line C++ for the statements of `program` (one element)."""
    lines = []
    for s in program:
        if skip(s):
            continue
        expr, pre = stmt_expr(s, value_of, dtypes)
        lines.extend(indent + p for p in pre)
        lines.append(f"{indent}const {P.ctype(_compute_dtype(s.dtype))} {s.var} = {expr};")
    return lines


def _strided_map_kernel(kernel: P.MapKernel, fn: P.TensorFunction, src: _Source) -> dict:
    """A map whose operands include strided views (transposes, slices, a part of a concat):
    one thread per element of the frame, each operand indexed through its offset and strides
    (contiguous operands through their row-major strides), NumPy broadcasting right-aligned.
    The bound symbols are kernel arguments here: view strides may name them."""
    params_by_name = {p.name: p for p in fn.params}
    frame = kernel.shape
    rank = len(frame)
    dims = P.spell_dims(frame)
    dtypes = {s.var: s.dtype for s in kernel.program}
    scalars = _scalar_params(kernel.program, params_by_name)
    status = needs_status(kernel.program)
    symbols = [b.symbol for b in fn.bindings]
    extra = (["int64_t n"] + [f"int64_t sym_{s}" for s in symbols]
             + [f"{P.ctype(t)} p_{n}" for n, t in scalars] + ["int32_t* status"])
    name = kernel.name
    operands = list(kernel.inputs) + [o.operand for o in kernel.outputs]
    L = [f"static __global__ void __launch_bounds__({THREADS}) {name}_s("
         + ", ".join(_kernel_params(kernel, extra)) + ") {"]
    L.append("  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;"
             " e += (int64_t)gridDim.x * blockDim.x) {")
    L.append("    int64_t rest = e; (void)rest;")
    for d in reversed(range(rank)):
        if frame[d] == 1:
            L.append(f"    const int64_t i{d} = 0;")
        else:
            L.append(f"    const int64_t i{d} = rest % {dims[d]}; rest /= {dims[d]};")
    for k, operand in enumerate(operands):
        shape = tuple(operand.shape)
        if len(shape) > rank:
            raise ValueError(f"{shape} does not broadcast to {frame}")
        offset, strides = operand.view if operand.view is not None else (
            0, P.contiguous_strides(shape))
        at = offset
        for j, dim in enumerate(shape):
            d = j + rank - len(shape)
            if dim == 1:
                continue  # a unit axis: index 0 (or broadcast over the frame)
            if dim != frame[d]:
                raise ValueError(f"{shape} does not broadcast to {frame}")
            at = P.term_add(at, P.term_mul(f"i{d}", strides[j]))
        L.append(f"    const int64_t at{k} = {P.spell_term(at)};")
    n_in = len(kernel.inputs)
    for s in kernel.program:
        if s.op == "input":
            i = s.args[0]
            load = f"in{i}[at{i}]"
            if kernel.inputs[i].dtype == "bf16":
                load = f"ppyb200::convert<float, __nv_bfloat16>({load})"
            L.append(f"    const {P.ctype(_compute_dtype(s.dtype))} {s.var} = {load};")
            continue
        expr, pre = stmt_expr(s, lambda v: v, dtypes)
        L.extend("    " + p for p in pre)
        L.append(f"    const {P.ctype(_compute_dtype(s.dtype))} {s.var} = {expr};")
    for j, out in enumerate(kernel.outputs):
        ct = P.ctype(out.operand.dtype)
        L.append(f"    out{j}[at{n_in + j}] = ppyb200::convert<{ct}, "
                 f"{P.ctype(_compute_dtype(dtypes[out.var]))}>({out.var});")
    L.append("  }")
    L.append("}")
    src.kernels.append("\n".join(L))
    args = ([o.pointer for o in kernel.inputs] + [o.operand.pointer for o in kernel.outputs]
            + ["n"] + [f"sym_{s}" for s in symbols] + [f"p_{n}" for n, _ in scalars]
            + ["status"])
    lines = ["{", f"  const int64_t n = {P.spell_count(frame)};", "  if (n > 0) {",
             f"    {name}_s<<<(unsigned)ppyb200_blocks(n, {THREADS}), {THREADS}, 0, stream>>>("
             + ", ".join(args) + ");",
             "    launches++;", "  }", "}"]
    return {"launch": lines, "status": status}


def _map_kernel(kernel: P.MapKernel, fn: P.TensorFunction, src: _Source) -> dict:
    """A flat or 2-D map: returns launch info for the host wrapper."""
    if any(o.view is not None for o in kernel.inputs) or any(
            o.operand.view is not None for o in kernel.outputs):
        return _strided_map_kernel(kernel, fn, src)
    params_by_name = {p.name: p for p in fn.params}
    frame = kernel.shape
    operand_shapes = [o.shape for o in kernel.inputs] + [o.operand.shape for o in kernel.outputs]
    flags = [presence(s, frame) for s in operand_shapes]
    dims, pres = coalesce(frame, flags)
    n_in = len(kernel.inputs)
    dtypes = {s.var: s.dtype for s in kernel.program}
    scalars = _scalar_params(kernel.program, params_by_name)
    status = needs_status(kernel.program)
    extra = ["int64_t n", "int64_t cols"] + [f"{P.ctype(t)} p_{n}" for n, t in scalars]
    extra.append("int32_t* status")
    rank = len(dims)
    sizes = [P.size_of(o.dtype) for o in kernel.inputs] + [P.size_of(o.operand.dtype)
                                                           for o in kernel.outputs]
    vec = 16 // max(sizes) if sizes else 4
    # Which operands vary along the last coalesced dim (vectorizable), and how.
    def cls(i):
        p = pres[i]
        if rank == 0:
            return "scalar"
        if rank == 1:
            return "elem" if p[0] else "scalar"
        if rank == 2:
            return {(True, True): "elem", (True, False): "rows", (False, True): "cols",
                    (False, False): "scalar"}[tuple(p)]
        return "general" if any(p) else "scalar"

    classes = [cls(i) for i in range(len(operand_shapes))]
    general = rank > 2
    name = kernel.name
    body_vec: list[str] = []
    body_scalar: list[str] = []

    def elem_index(c: str, e: str, row: str, col: str) -> str:
        return {"elem": e, "rows": row, "cols": col, "scalar": "0"}[c]

    # --- scalar kernel (any rank; also the tail and unaligned fallback)
    body_scalar.append(f"static __global__ void __launch_bounds__({THREADS}) {name}_s("
                       + ", ".join(_kernel_params(kernel, extra)) + ") {")
    body_scalar.append("  (void)cols;")
    body_scalar.append("  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;"
                       " e += (int64_t)gridDim.x * blockDim.x) {")
    if general:
        # unravel over the coalesced dims
        body_scalar.append("    int64_t rest = e;")
        for d in reversed(range(rank)):
            body_scalar.append(f"    const int64_t i{d} = rest % ({dim_expr(dims[d])}); "
                               f"rest /= ({dim_expr(dims[d])});")
        for k in range(len(operand_shapes)):
            terms = []
            stride = []
            for d in reversed(range(rank)):
                if pres[k][d]:
                    terms.append(f"i{d}" + "".join(f" * {x}" for x in stride))
                    stride.append(f"({dim_expr(dims[d])})")
            body_scalar.append(f"    const int64_t at{k} = {' + '.join(terms) if terms else '0'};")
    else:
        body_scalar.append("    const int64_t row = cols > 0 ? e / cols : 0; "
                           "const int64_t col = e - row * cols; (void)row; (void)col;")
        for k in range(len(operand_shapes)):
            body_scalar.append(f"    const int64_t at{k} = {elem_index(classes[k], 'e', 'row', 'col')};")

    def scalar_value(var):
        return var

    for i in range(n_in):
        ct = P.ctype(kernel.inputs[i].dtype)
        body_scalar.append(f"    const {ct} x{i} = in{i}[at{i}];")

    def value_s(v):
        stmt = next((s for s in kernel.program if s.var == v), None)
        return v if stmt is None or stmt.op != "input" else v

    for s in kernel.program:
        if s.op == "input":
            src_dtype = kernel.inputs[s.args[0]].dtype
            cdt = _compute_dtype(s.dtype)
            load = f"x{s.args[0]}"
            if src_dtype == "bf16":
                load = f"ppyb200::convert<float, __nv_bfloat16>({load})"
            body_scalar.append(f"    const {P.ctype(cdt)} {s.var} = {load};")
            continue
        expr, pre = stmt_expr(s, value_s, dtypes)
        body_scalar.extend("    " + p for p in pre)
        body_scalar.append(f"    const {P.ctype(_compute_dtype(s.dtype))} {s.var} = {expr};")
    for j, out in enumerate(kernel.outputs):
        k = n_in + j
        ct = P.ctype(out.operand.dtype)
        body_scalar.append(f"    out{j}[at{k}] = ppyb200::convert<{ct}, "
                           f"{P.ctype(_compute_dtype(dtypes[out.var]))}>({out.var});")
    body_scalar.append("  }")
    body_scalar.append("}")

    vectorizable = not general and rank >= 1 and vec > 1
    if vectorizable:
        u = MAP_UNROLL
        bounds = f"{THREADS}, {MAP_MIN_BLOCKS}" if MAP_MIN_BLOCKS else f"{THREADS}"
        body_vec.append(f"static __global__ void __launch_bounds__({bounds}) {name}_v("
                        + ", ".join(_kernel_params(kernel, extra)) + ") {")
        body_vec.append(f"  constexpr int VEC = {vec};")
        body_vec.append("  const int64_t nvec = n / VEC; (void)cols;")
        body_vec.append(f"  const int64_t stride = (int64_t)gridDim.x * blockDim.x * {u};")
        body_vec.append(f"  for (int64_t base = (int64_t)blockIdx.x * blockDim.x * {u} + threadIdx.x;"
                        " base < nvec; base += stride) {")
        # load phase: all vectors of all inputs first
        for r in range(u):
            body_vec.append(f"    const int64_t q{r} = base + (int64_t){r} * blockDim.x;")
            body_vec.append(f"    const bool ok{r} = q{r} < nvec;")
            body_vec.append(f"    const int64_t e{r} = q{r} * VEC;")
            if rank == 2:
                body_vec.append(f"    const int64_t row{r} = e{r} / cols; const int64_t col{r} = "
                                f"e{r} - row{r} * cols; (void)row{r}; (void)col{r};")
            for i, operand in enumerate(kernel.inputs):
                ct = P.ctype(operand.dtype)
                c = classes[i]
                if c == "elem":
                    body_vec.append(f"    ppyb200::Vec<{ct}, VEC> x{i}_{r}; if (ok{r}) x{i}_{r} = "
                                    f"ppyb200::load_vec_stream<{ct}, VEC>(in{i} + e{r});")
                elif c == "cols":
                    body_vec.append(f"    ppyb200::Vec<{ct}, VEC> x{i}_{r}; if (ok{r}) x{i}_{r} = "
                                    f"ppyb200::load_vec_cached<{ct}, VEC>(in{i} + col{r});")
                elif c == "rows":
                    body_vec.append(f"    {ct} x{i}_{r}{{}}; if (ok{r}) x{i}_{r} = __ldg(in{i} + row{r});")
                else:
                    body_vec.append(f"    const {ct} x{i}_{r} = in{i}[0];")
        for r in range(u):
            body_vec.append(f"    if (ok{r}) {{")
            for j, out in enumerate(kernel.outputs):
                ct = P.ctype(out.operand.dtype)
                body_vec.append(f"      ppyb200::Vec<{ct}, VEC> y{j};")
            body_vec.append("      #pragma unroll")
            body_vec.append("      for (int u = 0; u < VEC; ++u) {")
            for s in kernel.program:
                if s.op == "input":
                    i = s.args[0]
                    c = classes[i]
                    src_dtype = kernel.inputs[i].dtype
                    load = f"x{i}_{r}.v[u]" if c in ("elem", "cols") else f"x{i}_{r}"
                    if src_dtype == "bf16":
                        load = f"ppyb200::convert<float, __nv_bfloat16>({load})"
                    cdt = _compute_dtype(s.dtype)
                    body_vec.append(f"        const {P.ctype(cdt)} {s.var} = {load};")
                    continue
                expr, pre = stmt_expr(s, lambda v: v, dtypes)
                body_vec.extend("        " + p for p in pre)
                body_vec.append(f"        const {P.ctype(_compute_dtype(s.dtype))} {s.var} = {expr};")
            for j, out in enumerate(kernel.outputs):
                ct = P.ctype(out.operand.dtype)
                body_vec.append(f"        y{j}.v[u] = ppyb200::convert<{ct}, "
                                f"{P.ctype(_compute_dtype(dtypes[out.var]))}>({out.var});")
            body_vec.append("      }")
            for j, out in enumerate(kernel.outputs):
                ct = P.ctype(out.operand.dtype)
                body_vec.append(f"      ppyb200::store_vec_stream<{ct}, VEC>(out{j} + e{r}, y{j});")
            body_vec.append("    }")
        body_vec.append("  }")
        body_vec.append("}")
    src.kernels.append("\n".join(body_scalar))
    if vectorizable:
        src.kernels.append("\n".join(body_vec))
    # host-side launch code
    total = P.spell_count(frame)
    last = dim_expr(dims[-1]) if rank >= 1 else "(int64_t)1"
    args_in = [o.pointer for o in kernel.inputs]
    args_out = [o.operand.pointer for o in kernel.outputs]
    arg_scalars = [f"p_{n}" for n, _ in scalars]
    call_args = ", ".join(args_in + args_out + ["n", "cols"] + arg_scalars + ["status"])
    lines = ["{", f"  const int64_t n = {total};", f"  const int64_t cols = {last};",
             "  if (n > 0) {"]
    if vectorizable:
        aligned = " && ".join(
            [f"ppyb200_aligned({p}, {vec * P.size_of(o.dtype)})"
             for p, o, c in zip(args_in, kernel.inputs, classes) if c in ("elem", "cols")]
            + [f"ppyb200_aligned({p}, {vec * P.size_of(o.operand.dtype)})"
               for p, o in zip(args_out, kernel.outputs)]
            or ["true"])
        cond = f"(n % {vec} == 0) && (cols % {vec} == 0) && {aligned}" if rank == 2 else (
            f"{aligned}")
        lines += [f"    if ({cond}) {{",
                  f"      const int64_t nvec = n / {vec};",
                  f"      const int64_t blocks = ppyb200_blocks(nvec, {THREADS} * {MAP_UNROLL});",
                  f"      {name}_v<<<(unsigned)blocks, {THREADS}, 0, stream>>>({call_args});",
                  "      launches++;"]
        if rank == 1:
            lines += [f"      const int64_t done = nvec * {vec};",
                      "      if (done < n) {",
                      "        /* the ragged tail: the scalar kernel over the last elements */",
                      f"        {name}_tail(" + ", ".join(args_in + args_out) + ", done, n"
                      + "".join(", " + a for a in arg_scalars) + ", status, stream);",
                      "        launches++;",
                      "      }"]
        lines += ["    } else {",
                  f"      {name}_s<<<(unsigned)ppyb200_blocks(n, {THREADS}), {THREADS}, 0, stream>>>({call_args});",
                  "      launches++;",
                  "    }"]
    else:
        lines += [f"    {name}_s<<<(unsigned)ppyb200_blocks(n, {THREADS}), {THREADS}, 0, stream>>>({call_args});",
                  "    launches++;"]
    lines += ["  }", "}"]
    if vectorizable and rank == 1:
        # A tail launcher: the scalar kernel with the pointers advanced to `done`.
        tparams = ([f"const {P.ctype(o.dtype)}* in{i}" for i, o in enumerate(kernel.inputs)]
                   + [f"{P.ctype(o.operand.dtype)}* out{j}" for j, o in enumerate(kernel.outputs)]
                   + ["int64_t done", "int64_t n"]
                   + [f"{P.ctype(t)} p_{nm}" for nm, t in scalars]
                   + ["int32_t* status", "cudaStream_t stream"])
        adv = []
        for i, c in enumerate(classes[:n_in]):
            adv.append(f"in{i} + done" if c == "elem" else f"in{i}")
        for j in range(len(kernel.outputs)):
            adv.append(f"out{j} + done")
        targs = ", ".join(adv + ["n - done", "(int64_t)1"] + [f"p_{nm}" for nm, _ in scalars]
                          + ["status"])
        src.kernels.append(
            f"static void {name}_tail({', '.join(tparams)}) {{\n"
            f"  {name}_s<<<1, {THREADS}, 0, stream>>>({targs});\n}}")
    return {"launch": lines, "status": status}


def _row_layout(kernel: P.RowKernel) -> dict:
    sizes = [P.size_of(o.dtype) for o in kernel.inputs] + [P.size_of(o.operand.dtype)
                                                           for o in kernel.outputs]
    vec = 16 // max(sizes) if sizes else 4
    if kernel.cols % vec:
        vec = 1
    chunks = kernel.cols // vec
    tpr = 1
    while tpr * 2 <= min(chunks, 32):
        tpr *= 2
    nch = -(-chunks // tpr)
    if nch * vec > 32 and chunks > 32:
        tpr = 32
        while -(-chunks // tpr) * vec > 32 and tpr < 1024:
            tpr *= 2
        nch = -(-chunks // tpr)
    block = ROW_THREADS if tpr <= 32 else tpr
    return {"vec": vec, "chunks": chunks, "tpr": tpr, "nch": nch, "block": block,
            "rows_per_block": block // tpr if tpr <= 32 else 1}


def _row_kernel(kernel: P.RowKernel, fn: P.TensorFunction, src: _Source) -> dict:
    params_by_name = {p.name: p for p in fn.params}
    layout = _row_layout(kernel)
    vec, tpr, nch, block = layout["vec"], layout["tpr"], layout["nch"], layout["block"]
    chunks = layout["chunks"]
    frame = kernel.shape
    rows_shape = frame[: len(frame) - kernel.reduced]
    # class of every input: elem / rows / cols / scalar
    row_rank = len(rows_shape)

    def classify(shape: tuple) -> str:
        flags = presence(shape, frame)
        lead = any(flags[:row_rank])
        trail = any(flags[row_rank:])
        if lead and trail:
            if not all(f or d == 1 for f, d in zip(flags, frame)):
                raise ValueError(f"{shape} is partly broadcast over {frame}")
            return "elem"
        if lead:
            if not all(f or d == 1 for f, d in zip(flags[:row_rank], frame[:row_rank])):
                raise ValueError(f"{shape} is partly broadcast over the rows of {frame}")
            return "rows"
        if trail:
            if not all(f or d == 1 for f, d in zip(flags[row_rank:], frame[row_rank:])):
                raise ValueError(f"{shape} is partly broadcast over a row of {frame}")
            return "cols"
        return "scalar"

    in_class = [classify(o.shape) for o in kernel.inputs]
    # statement classes
    cls: dict[str, str] = {}
    order = {"scalar": 0, "rows": 1, "cols": 1, "elem": 2}
    for s in kernel.program:
        if s.op == "input":
            cls[s.var] = in_class[s.args[0]]
        elif s.op in ("const", "param"):
            cls[s.var] = "scalar"
        elif s.op == "reduce":
            cls[s.var] = "rows"
        else:
            cs = [cls[a] for a in s.args]
            if "elem" in cs or ("rows" in cs and "cols" in cs):
                cls[s.var] = "elem"
            elif "rows" in cs:
                cls[s.var] = "rows"
            elif "cols" in cs:
                cls[s.var] = "cols"
            else:
                cls[s.var] = "scalar"
    out_class = []
    for out in kernel.outputs:
        c = cls[out.var]
        oc = classify(out.operand.shape) if out.operand.shape != rows_shape else "rows"
        if c == "elem" and oc != "elem":
            raise ValueError("an element value stored into a smaller tensor")
        out_class.append(oc if c != "scalar" else oc)
    dtypes = {s.var: s.dtype for s in kernel.program}
    scalars = _scalar_params(kernel.program, params_by_name)
    extra = ["int64_t R"] + [f"{P.ctype(t)} p_{n}" for n, t in scalars] + ["int32_t* status"]
    name = kernel.name
    n_red = sum(1 for s in kernel.program if s.op == "reduce")
    warps = block // 32
    masked = chunks % tpr != 0
    elem_inputs = [i for i, c in enumerate(in_class) if c == "elem"]
    # Pipelined form: persistent warps, each prefetching its next row groups into a ring in
    # shared memory (bulk copies completing on an mbarrier per stage) while it computes the
    # current one. It needs 16-byte chunks and a row group per warp (rows of at most 32
    # lanes). A stage whose copy never completes (bounded wait) raises the status word when
    # the call has one.
    pipelined = tpr <= 32 and elem_inputs and all(
        vec * P.size_of(kernel.inputs[i].dtype) == 16 for i in elem_inputs)
    rpw = 32 // tpr if tpr <= 32 else 1
    seg = {}
    buf_bytes = 0
    for i in elem_inputs:
        seg[i] = buf_bytes
        buf_bytes += rpw * kernel.cols * P.size_of(kernel.inputs[i].dtype)
        buf_bytes = (buf_bytes + 15) // 16 * 16
    stages = ROW_STAGES
    while stages > 2 and warps * stages * buf_bytes > ROW_SMEM_LIMIT:
        stages -= 1
    smem_bytes = warps * stages * buf_bytes
    if smem_bytes > ROW_SMEM_LIMIT:
        pipelined = False
    bounds = f"{block}, {ROW_MIN_BLOCKS}" if ROW_MIN_BLOCKS else f"{block}"
    L = [f"static __global__ void __launch_bounds__({bounds}) {name}("
         + ", ".join(_kernel_params(kernel, extra)) + ") {"]
    L.append(f"  constexpr int VEC = {vec}, TPR = {tpr}, NCH = {nch}, CHUNKS = {chunks}, "
             f"COLS = {kernel.cols};")
    L.append("  (void)CHUNKS; (void)status;")
    # launched with the programmatic-serialization attribute (ppyb200::launch_pdl): wait
    # for the previous kernel's results, and let the next kernel's CTAs start setting up
    L.append("  ppyb200::pdl_wait();")
    L.append("  ppyb200::pdl_trigger();")
    if tpr <= 32:
        L.append("  const int lane = threadIdx.x % TPR;")
        L.append(f"  const int64_t slot = (threadIdx.x & 31) / TPR; constexpr int64_t RPW = 32 / TPR;")
    else:
        L.append("  const int lane = threadIdx.x; const int64_t slot = 0;")
        if n_red:
            L.append(f"  __shared__ float red_f[{max(n_red, 1)}][{warps}];")
            L.append(f"  __shared__ double red_d[{max(n_red, 1)}][{warps}];")
            L.append(f"  __shared__ int64_t red_i[{max(n_red, 1)}][{warps}];")
    for i, operand in enumerate(kernel.inputs):
        ct = P.ctype(operand.dtype)
        if in_class[i] == "scalar":
            L.append(f"  const {ct} s{i} = in{i}[0];")

    def value(var: str, where: str) -> str:
        c = cls[var]
        if c in ("elem", "cols"):
            return f"{var}[j][u]" if where == "elem" else var
        return var

    def input_expr(s: P.Stmt, where: str) -> str:
        i = s.args[0]
        c = in_class[i]
        ct_i = P.ctype(kernel.inputs[i].dtype)
        if c == "elem":
            if pipelined:
                e = (f"reinterpret_cast<const ppyb200::Vec<{ct_i}, VEC>*>(buf + {seg[i]} + "
                     f"(int64_t)slot * COLS * {P.size_of(kernel.inputs[i].dtype)})[j * TPR + lane].v[u]")
            else:
                e = f"x{i}[j].v[u]"
        elif c == "cols":
            # per-column vectors (gamma, bias...) are read where they are used, from L1/L2
            e = f"ppyb200::load_vec_cached<{ct_i}, VEC>(in{i} + (int64_t)(j * TPR + lane) * VEC).v[u]"
        elif c == "rows":
            e = f"r{i}"
        else:
            e = f"s{i}"
        if masked and c in ("elem", "cols"):
            # a lane past the row's last chunk reads nothing (its values are never folded or
            # stored, but the read itself would leave the row: past a staged row group's
            # shared memory, or past the end of a column vector)
            e = f"((j * TPR + lane < CHUNKS) ? {e} : {ct_i}{{}})"
        if kernel.inputs[i].dtype == "bf16":
            e = f"ppyb200::convert<float, __nv_bfloat16>({e})"
        return e

    # statements over scalars only are computed once per thread
    for s in kernel.program:
        if cls[s.var] != "scalar":
            continue
        ct = P.ctype(_compute_dtype(s.dtype))
        if s.op == "input":
            L.append(f"  const {ct} {s.var} = {input_expr(s, 'scalar')};")
        else:
            expr, pre = stmt_expr(s, lambda v: v, dtypes)
            L.extend("  " + p for p in pre)
            L.append(f"  const {ct} {s.var} = {expr};")
    # the body over one row (`row`, `active` and, when pipelined, `buf` in scope)
    B = []
    if not pipelined:
        for i in elem_inputs:
            ct = P.ctype(kernel.inputs[i].dtype)
            B.append(f"ppyb200::Vec<{ct}, VEC> x{i}[NCH];")
            B.append("#pragma unroll")
            B.append("for (int j = 0; j < NCH; ++j) {")
            guard = "active && (j * TPR + lane < CHUNKS)" if masked else "active"
            B.append(f"  if ({guard}) x{i}[j] = ppyb200::load_vec_stream<{ct}, VEC>("
                     f"in{i} + row * COLS + (int64_t)(j * TPR + lane) * VEC);")
            B.append(f"  else {{ for (int u = 0; u < VEC; ++u) x{i}[j].v[u] = {ct}{{}}; }}")
            B.append("}")
    for i, operand in enumerate(kernel.inputs):
        if in_class[i] == "rows":
            ct = P.ctype(operand.dtype)
            B.append(f"const {ct} r{i} = active ? in{i}[row] : {ct}{{}};")
    red_index = 0
    for s in kernel.program:
        c = cls[s.var]
        if c == "scalar":
            continue
        ct = P.ctype(_compute_dtype(s.dtype))
        if s.op == "reduce":
            kind = s.attrs["kind"]
            arg = s.args[0]
            acc = f"{s.var}_acc"
            B.append(f"{ct} {acc} = {identity_literal(kind, _compute_dtype(s.dtype))};")
            if cls[arg] in ("elem", "cols"):
                B.append("#pragma unroll")
                B.append("for (int j = 0; j < NCH; ++j) {")
                guard = "active && (j * TPR + lane < CHUNKS)" if masked else "active"
                B.append(f"  if ({guard}) {{")
                B.append("    #pragma unroll")
                B.append("    for (int u = 0; u < VEC; ++u) "
                         f"{acc} = {combine_expr(kind, acc, value(arg, 'elem'))};")
                B.append("  }")
                B.append("}")
            else:
                # a fold over COLS copies of one value per row (a reduce of a row scalar)
                B.append("if (active) {")
                B.append("  for (int j = 0; j < NCH; ++j) if (j * TPR + lane < CHUNKS) "
                         f"for (int u = 0; u < VEC; ++u) {acc} = {combine_expr(kind, acc, arg)};")
                B.append("}")
            op = _COMBINE[kind]
            if tpr <= 32:
                B.append(f"const {ct} {s.var} = ppyb200::group_reduce<{op}, TPR>({acc});")
            else:
                smem = {"float": "red_f", "double": "red_d"}.get(ct, "red_i")
                smem_t = {"red_f": "float", "red_d": "double"}.get(smem, "int64_t")
                B.append(f"{acc} = ppyb200::group_reduce<{op}, 32>({acc});")
                B.append(f"if ((threadIdx.x & 31) == 0) {smem}[{red_index}][threadIdx.x >> 5] = ({smem_t}){acc};")
                B.append("__syncthreads();")
                B.append(f"{ct} {s.var} = ({ct}){smem}[{red_index}][0];")
                B.append(f"for (int w = 1; w < {warps}; ++w) {s.var} = {combine_expr(kind, s.var, f'({ct}){smem}[{red_index}][w]')};")
            red_index += 1
            continue
        if c == "rows":
            if s.op == "input":
                B.append(f"const {ct} {s.var} = {input_expr(s, 'rows')};")
            else:
                expr, pre = stmt_expr(s, lambda v: v, dtypes)
                B.extend(pre)
                B.append(f"const {ct} {s.var} = {expr};")
            continue
        # elem and cols statements: one value per element of this lane's chunks
        f32_row_divide = (s.op == "div" and _compute_dtype(s.dtype) == "f32"
                          and cls[s.args[1]] in ("rows", "scalar"))
        if f32_row_divide:
            # an f32 division by one value per row: its reciprocal once per row, then a
            # multiply per element (within an ulp and a half of the division)
            B.append(f"const {ct} {s.var}_rcp = {ct}(1) / {s.args[1]};")
        B.append(f"{ct} {s.var}[NCH][VEC];")
        B.append("#pragma unroll")
        B.append("for (int j = 0; j < NCH; ++j) {")
        B.append("  #pragma unroll")
        B.append("  for (int u = 0; u < VEC; ++u) {")
        if s.op == "input":
            B.append(f"    {s.var}[j][u] = {input_expr(s, 'elem')};")
        elif f32_row_divide:
            B.append(f"    {s.var}[j][u] = {value(s.args[0], 'elem')} * {s.var}_rcp;")
        elif s.op == "math" and s.attrs["fn"] == "exp" and _compute_dtype(s.dtype) == "f32":
            # the SFU exponential (PTX ex2.approx after a scale by log2 e; CUDA's __expf):
            # within 2 + 1.16 |x| ulp, inside the f32 tolerance
            B.append(f"    {s.var}[j][u] = __expf({value(s.args[0], 'elem')});")
        else:
            expr, pre = stmt_expr(s, lambda v: value(v, "elem"), dtypes)
            B.extend("    " + p for p in pre)
            B.append(f"    {s.var}[j][u] = {expr};")
        B.append("  }")
        B.append("}")
    for j_out, (out, oc) in enumerate(zip(kernel.outputs, out_class)):
        ct = P.ctype(out.operand.dtype)
        src_ct = P.ctype(_compute_dtype(dtypes[out.var]))
        c = cls[out.var]
        if oc == "elem":
            B.append("if (active) {")
            B.append("  #pragma unroll")
            B.append("  for (int j = 0; j < NCH; ++j) {")
            if masked:
                B.append("    if (j * TPR + lane >= CHUNKS) continue;")
            B.append(f"    ppyb200::Vec<{ct}, VEC> y;")
            B.append("    #pragma unroll")
            B.append(f"    for (int u = 0; u < VEC; ++u) y.v[u] = ppyb200::convert<{ct}, {src_ct}>({value(out.var, 'elem') if c in ('elem', 'cols') else out.var});")
            B.append(f"    ppyb200::store_vec_stream<{ct}, VEC>(out{j_out} + row * COLS + (int64_t)(j * TPR + lane) * VEC, y);")
            B.append("  }")
            B.append("}")
        else:
            B.append(f"if (active && lane == 0) out{j_out}[row] = ppyb200::convert<{ct}, {src_ct}>({out.var});")
    if pipelined:
        L.append("  extern __shared__ __align__(16) unsigned char smem[];")
        L.append(f"  constexpr int64_t WPB = {warps}, BUF = {buf_bytes};")
        L.append("  const int64_t warp = threadIdx.x >> 5;")
        L.append("  const int64_t groups = (R + RPW - 1) / RPW;")
        L.append("  const int64_t first = (int64_t)blockIdx.x * WPB + warp;")
        L.append("  const int64_t stride = (int64_t)gridDim.x * WPB;")
        L.append(f"  constexpr int STAGES = {stages};")
        L.append("  unsigned char* wbuf = smem + warp * STAGES * BUF;")
        # the warp's ring: a row group (RPW consecutive rows, contiguous in every input) per
        # stage, one bulk copy per input, one mbarrier per stage
        L.append("  __shared__ uint64_t ring[WPB][STAGES];")
        L.append("  if ((threadIdx.x & 31) == 0) ppyb200::ring_init(ring[warp], STAGES);")
        L.append("  __syncwarp();")
        L.append("  uint32_t phases = 0;  // bit k: the parity stage k completes next")
        row_bytes = sum(P.size_of(kernel.inputs[i].dtype) for i in elem_inputs)
        P_ = ["  auto prefetch = [&](int64_t g, int b) {",
              "    const int64_t prow = g * RPW;",
              "    if (prow >= R || (threadIdx.x & 31) != 0) return;",
              "    const int64_t rows = R - prow < RPW ? R - prow : RPW;",
              "    unsigned char* pb = wbuf + b * BUF;",
              f"    ppyb200::ring_expect(&ring[warp][b], (uint32_t)(rows * COLS * {row_bytes}));"]
        for i in elem_inputs:
            size = P.size_of(kernel.inputs[i].dtype)
            P_.append(f"    ppyb200::ring_load(pb + {seg[i]}, in{i} + prow * COLS, "
                      f"(uint32_t)(rows * COLS * {size}), &ring[warp][b]);")
        P_.append("  };")
        L.extend(P_)
        # STAGES - 1 row groups in flight ahead of the one computed
        L.append("  #pragma unroll")
        L.append("  for (int k = 0; k < STAGES - 1; ++k)")
        L.append("    if (first + k * stride < groups) prefetch(first + k * stride, k);")
        L.append("  int b = 0;")
        L.append("  for (int64_t g = first; g < groups; g += stride, b = (b + 1) % STAGES) {")
        L.append("    const int64_t ahead = g + (STAGES - 1) * stride;")
        L.append("    __syncwarp();  // every lane has read the stage that is refilled next")
        L.append("    if (ahead < groups) prefetch(ahead, (b + STAGES - 1) % STAGES);")
        L.append("    ppyb200::ring_wait(&ring[warp][b], (phases >> b) & 1u, status);")
        L.append("    phases ^= 1u << b;")
        L.append("    const unsigned char* buf = wbuf + b * BUF;")
        L.append("    const int64_t row = g * RPW + slot;")
        L.append("    const bool active = row < R;")
        L.extend("    " + line for line in B)
        L.append("  }")
        L.append("}")
    else:
        L.append("  {")
        L.append(f"    constexpr int64_t RPB = {layout['rows_per_block']};")
        L.append("    const int64_t row = (int64_t)blockIdx.x * RPB + (threadIdx.x / TPR);"
                 if tpr <= 32 else "    const int64_t row = (int64_t)blockIdx.x;")
        L.append("    const bool active = row < R;")
        L.extend("    " + line for line in B)
        L.append("  }")
        L.append("}")
    src.kernels.append("\n".join(L))
    rows_count = P.spell_count(rows_shape)
    call_args = ", ".join([o.pointer for o in kernel.inputs] + [o.operand.pointer for o in kernel.outputs]
                          + ["R"] + [f"p_{n}" for n, _ in scalars] + ["status"])
    align_checks = [f"ppyb200_aligned({o.pointer}, {vec * P.size_of(o.dtype)})"
                    for o, c in zip(kernel.inputs, in_class) if c in ("elem", "cols")]
    align_checks += [f"ppyb200_aligned({o.operand.pointer}, {vec * P.size_of(o.operand.dtype)})"
                     for o, oc in zip(kernel.outputs, out_class) if oc == "elem"]
    lines = ["{", f"  const int64_t R = {rows_count};", "  if (R > 0) {"]
    if align_checks and vec > 1:
        lines.append(f"    if (!({' && '.join(align_checks)})) {{ ppyb200_set_error(\"{name}: "
                     f"row operands must be {vec * 4}-byte aligned\"); return PPY_STATUS_RAISED; }}")
    if pipelined:
        lines += [f"    static ppyb200::DeviceOnce resident_on;  // blocks of {name} one SM holds",
                  "    int resident = 0;",
                  "    const cudaError_t set_up = resident_on.get([](int* v) {",
                  f"      cudaError_t e = cudaFuncSetAttribute({name}, cudaFuncAttributeMaxDynamicSharedMemorySize, {smem_bytes});",
                  f"      if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(v, {name}, {block}, {smem_bytes});",
                  "      if (*v < 1) *v = 1;",
                  "      return e;",
                  "    }, &resident);",
                  f"    if (set_up != cudaSuccess) return ppyb200_check((int32_t)set_up, \"{name}: set-up\");",
                  f"    const int64_t groups = (R + {rpw} - 1) / {rpw};",
                  f"    int64_t blocks = (groups + {warps} - 1) / {warps};",
                  "    const int64_t cap = (int64_t)ppyb200_sm_count() * resident;",
                  "    if (blocks > cap) blocks = cap;",
                  f"    const cudaError_t launched = ppyb200::launch_pdl({name}, dim3((unsigned)blocks), dim3({block}), {smem_bytes}, stream, {call_args});",
                  f"    if (launched != cudaSuccess) return ppyb200_check((int32_t)launched, \"{name}\");",
                  "    launches++;", "  }", "}"]
    else:
        rpb = layout["rows_per_block"]
        lines += [f"    const int64_t blocks = (R + {rpb} - 1) / {rpb};",
                  f"    const cudaError_t launched = ppyb200::launch_pdl({name}, dim3((unsigned)blocks), dim3({block}), 0, stream, {call_args});",
                  f"    if (launched != cudaSuccess) return ppyb200_check((int32_t)launched, \"{name}\");",
                  "    launches++;", "  }", "}"]
    return {"launch": lines, "status": needs_status(kernel.program)}


def _reduce_all_kernel(kernel: P.ReduceAllKernel, fn: P.TensorFunction, src: _Source) -> dict:
    params_by_name = {p.name: p for p in fn.params}
    frame = kernel.shape
    flags = [presence(o.shape, frame) for o in kernel.inputs]
    dims, pres = coalesce(frame, flags)
    rank = len(dims)
    dtypes = {s.var: s.dtype for s in kernel.program}
    scalars = _scalar_params(kernel.program, params_by_name)
    acc_t = P.ctype(_compute_dtype(kernel.dtype))
    name = kernel.name
    kind = kernel.reduce
    op = _COMBINE[kind]
    ident = identity_literal(kind, _compute_dtype(kernel.dtype))
    extra = ["int64_t n"] + [f"{P.ctype(t)} p_{n}" for n, t in scalars] + [
        f"{acc_t}* __restrict__ partials", "int32_t* status"]
    params = [f"const {P.ctype(o.dtype)}* __restrict__ in{i}" for i, o in enumerate(kernel.inputs)]
    L = [f"static __global__ void __launch_bounds__({THREADS}) {name}_part(" + ", ".join(params + extra) + ") {",
         f"  {acc_t} acc = {ident};", "  (void)status;"]
    L.append("  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; "
             "e += (int64_t)gridDim.x * blockDim.x) {")
    # index of each input
    if rank <= 1:
        for i in range(len(kernel.inputs)):
            L.append(f"    const int64_t at{i} = {'e' if rank == 1 and pres[i][0] else '0'};")
    else:
        L.append("    int64_t rest = e;")
        for d in reversed(range(rank)):
            L.append(f"    const int64_t i{d} = rest % ({dim_expr(dims[d])}); rest /= ({dim_expr(dims[d])});")
        for k in range(len(kernel.inputs)):
            terms, stride = [], []
            for d in reversed(range(rank)):
                if pres[k][d]:
                    terms.append(f"i{d}" + "".join(f" * {x}" for x in stride))
                    stride.append(f"({dim_expr(dims[d])})")
            L.append(f"    const int64_t at{k} = {' + '.join(terms) if terms else '0'};")
    for s in kernel.program:
        ct = P.ctype(_compute_dtype(s.dtype))
        if s.op == "input":
            e = f"in{s.args[0]}[at{s.args[0]}]"
            if kernel.inputs[s.args[0]].dtype == "bf16":
                e = f"ppyb200::convert<float, __nv_bfloat16>({e})"
            L.append(f"    const {ct} {s.var} = {e};")
            continue
        expr, pre = stmt_expr(s, lambda v: v, dtypes)
        L.extend("    " + p for p in pre)
        L.append(f"    const {ct} {s.var} = {expr};")
    L.append(f"    acc = {op}::apply(acc, ({acc_t}){kernel.var});")
    L.append("  }")
    L += _block_reduce_lines(acc_t, op, "acc")
    L.append("  if (threadIdx.x == 0) partials[blockIdx.x] = acc;")
    L.append("}")
    out_ct = P.ctype(kernel.output.dtype)
    L2 = [f"static __global__ void __launch_bounds__({THREADS}) {name}_fin(const {acc_t}* __restrict__ partials, "
          f"int64_t parts, {out_ct}* __restrict__ out0) {{",
          f"  {acc_t} acc = {ident};",
          "  for (int64_t i = threadIdx.x; i < parts; i += blockDim.x) "
          f"acc = {op}::apply(acc, partials[i]);"]
    L2 += _block_reduce_lines(acc_t, op, "acc")
    L2.append(f"  if (threadIdx.x == 0) out0[0] = ppyb200::convert<{out_ct}, {acc_t}>(acc);")
    L2.append("}")
    src.kernels.append("\n".join(L))
    src.kernels.append("\n".join(L2))
    call = ", ".join([o.pointer for o in kernel.inputs] + ["n"] + [f"p_{n}" for n, _ in scalars]
                     + [f"({acc_t}*)part", "status"])
    lines = ["{", f"  const int64_t n = {P.spell_count(frame)};",
             f"  const int64_t parts = ppyb200_reduce_blocks(n, {THREADS});",
             f"  void* part = ppyb200_scratch_take(&scratch, parts * (int64_t)sizeof({acc_t}));",
             "  if (part == nullptr) return PPY_STATUS_RAISED;",
             f"  {name}_part<<<(unsigned)parts, {THREADS}, 0, stream>>>({call});",
             f"  {name}_fin<<<1, {THREADS}, 0, stream>>>(({acc_t}*)part, parts, {kernel.output.pointer});",
             "  launches += 2;", "}"]
    scratch = (f"ppyb200_round256(ppyb200_reduce_blocks({P.spell_count(frame)}, {THREADS}) * "
               f"(int64_t)sizeof({acc_t}))")
    return {"launch": lines, "status": needs_status(kernel.program), "scratch": scratch}


def _block_reduce_lines(acc_t: str, op: str, acc: str) -> list[str]:
    """Fold every thread's `acc` into thread 0's, warps first, then in warp order."""
    return [f"  {acc} = ppyb200::group_reduce<{op}, 32>({acc});",
            f"  __shared__ {acc_t} warp_acc[{THREADS // 32}];",
            f"  if ((threadIdx.x & 31) == 0) warp_acc[threadIdx.x >> 5] = {acc};",
            "  __syncthreads();",
            "  if (threadIdx.x == 0) {",
            f"    {acc} = warp_acc[0];",
            f"    for (int w = 1; w < {THREADS // 32}; ++w) {acc} = {op}::apply({acc}, warp_acc[w]);",
            "  }"]


def _reduce_cols_kernel(kernel: P.ReduceColsKernel, fn: P.TensorFunction, src: _Source) -> dict:
    params_by_name = {p.name: p for p in fn.params}
    frame = kernel.shape
    lead = frame[: kernel.reduced]
    trail = frame[kernel.reduced:]
    dtypes = {s.var: s.dtype for s in kernel.program}
    scalars = _scalar_params(kernel.program, params_by_name)
    acc_t = P.ctype(_compute_dtype(kernel.dtype))
    kind = kernel.reduce
    op = _COMBINE[kind]
    ident = identity_literal(kind, _compute_dtype(kernel.dtype))
    name = kernel.name

    def cls(shape):
        flags = presence(shape, frame)
        a, b = any(flags[: kernel.reduced]), any(flags[kernel.reduced:])
        return {(True, True): "elem", (True, False): "rows", (False, True): "cols",
                (False, False): "scalar"}[(a, b)]

    classes = [cls(o.shape) for o in kernel.inputs]
    params = [f"const {P.ctype(o.dtype)}* __restrict__ in{i}" for i, o in enumerate(kernel.inputs)]
    extra = ["int64_t R", "int64_t C", "int64_t rows_per_chunk"] + [
        f"{P.ctype(t)} p_{n}" for n, t in scalars] + [f"{acc_t}* __restrict__ partials", "int32_t* status"]
    L = [f"static __global__ void __launch_bounds__({THREADS}) {name}_part(" + ", ".join(params + extra) + ") {",
         "  (void)status;",
         "  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;",
         "  if (c >= C) return;",
         "  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;",
         "  const int64_t r1 = r0 + rows_per_chunk < R ? r0 + rows_per_chunk : R;",
         f"  {acc_t} acc = {ident};",
         "  for (int64_t r = r0; r < r1; ++r) {"]
    for s in kernel.program:
        ct = P.ctype(_compute_dtype(s.dtype))
        if s.op == "input":
            i = s.args[0]
            idx = {"elem": "r * C + c", "rows": "r", "cols": "c", "scalar": "0"}[classes[i]]
            e = f"in{i}[{idx}]"
            if kernel.inputs[i].dtype == "bf16":
                e = f"ppyb200::convert<float, __nv_bfloat16>({e})"
            L.append(f"    const {ct} {s.var} = {e};")
            continue
        expr, pre = stmt_expr(s, lambda v: v, dtypes)
        L.extend("    " + p for p in pre)
        L.append(f"    const {ct} {s.var} = {expr};")
    L.append(f"    acc = {op}::apply(acc, ({acc_t}){kernel.var});")
    L.append("  }")
    L.append("  partials[(int64_t)blockIdx.y * C + c] = acc;")
    L.append("}")
    out_ct = P.ctype(kernel.output.dtype)
    L2 = [f"static __global__ void __launch_bounds__({THREADS}) {name}_fin(const {acc_t}* __restrict__ partials, "
          f"int64_t chunks, int64_t C, {out_ct}* __restrict__ out0) {{",
          "  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;",
          "  if (c >= C) return;",
          f"  {acc_t} acc = {ident};",
          f"  for (int64_t k = 0; k < chunks; ++k) acc = {op}::apply(acc, partials[k * C + c]);",
          f"  out0[c] = ppyb200::convert<{out_ct}, {acc_t}>(acc);",
          "}"]
    src.kernels.append("\n".join(L))
    src.kernels.append("\n".join(L2))
    call = ", ".join([o.pointer for o in kernel.inputs] + ["R", "C", "rows_per_chunk"]
                     + [f"p_{n}" for n, _ in scalars] + [f"({acc_t}*)part", "status"])
    lines = ["{", f"  const int64_t R = {P.spell_count(lead)};", f"  const int64_t C = {P.spell_count(trail)};",
             "  if (C > 0) {",
             f"    const int64_t col_blocks = (C + {THREADS} - 1) / {THREADS};",
             "    int64_t chunks = ppyb200_col_chunks(R, col_blocks);",
             "    const int64_t rows_per_chunk = R > 0 ? (R + chunks - 1) / chunks : 1;",
             "    chunks = R > 0 ? (R + rows_per_chunk - 1) / rows_per_chunk : 1;",
             f"    void* part = ppyb200_scratch_take(&scratch, chunks * C * (int64_t)sizeof({acc_t}));",
             "    if (part == nullptr) return PPY_STATUS_RAISED;",
             f"    {name}_part<<<dim3((unsigned)col_blocks, (unsigned)chunks), {THREADS}, 0, stream>>>({call});",
             f"    {name}_fin<<<(unsigned)col_blocks, {THREADS}, 0, stream>>>(({acc_t}*)part, chunks, C, {kernel.output.pointer});",
             "    launches += 2;", "  }", "}"]
    lead_n, trail_n = P.spell_count(lead), P.spell_count(trail)
    scratch = (f"ppyb200_round256((ppyb200_col_chunks({lead_n}, ({trail_n} + {THREADS} - 1) / {THREADS}) + 1)"
               f" * ({trail_n}) * (int64_t)sizeof({acc_t}))")
    return {"launch": lines, "status": needs_status(kernel.program), "scratch": scratch}


# -- host wrappers ------------------------------------------------------------------------


def _abi_params(params: list) -> list[str]:
    atoms = []
    for p in params:
        if p.kind == "buffer":
            atoms.append(f"{P.ctype(p.dtype)}* {p.name}_ptr")
            atoms.append(f"int64_t {p.name}_len")
        elif p.kind == "ptr":
            atoms.append(f"{P.ctype(p.dtype)}* {p.name}")
        else:
            atoms.append(f"{P.ctype(p.dtype)} p_{p.name}")
    return atoms


#: Elements per slice of a pipelined host-memory call (8 MB of f32 per operand).
PIPELINE_SLICE = 1 << 21


def _slices(fn: P.TensorFunction, buffers: list, counts: dict) -> tuple[str, dict] | None:
    """How a function splits into independent slices along its one symbolic length: one
    binding of a symbol R from a buffer's length, no temporaries, every kernel a map over [R]
    or a row kernel over [R, C] of contiguous (not viewed) operands. Every buffer then holds
    k * R elements for a constant k (k elements per index of R: 1 for a map, C for the rows of
    a row kernel, 1 for a per-row result), and slices [r0, r0 + len) of R touch elements
    [k r0, k (r0 + len)) of it only; or a constant count (a per-column operand such as a
    layernorm's gamma), which every slice reads whole and no kernel writes. Returns ("sym_R",
    {buffer: k, or None for a whole one}); None when the function does not split so."""
    if len(fn.bindings) != 1 or fn.temps or fn.dim_guards or not fn.kernels or not buffers:
        return None
    b = fn.bindings[0]
    r = b.symbol
    for kernel in fn.kernels:
        if kernel.kind not in ("map", "row"):
            return None
        shape = tuple(kernel.shape)
        if kernel.kind == "map" and shape != (r,):
            return None
        if kernel.kind == "row" and (len(shape) != 2 or shape[0] != r
                                     or not isinstance(shape[1], int)):
            return None
        operands = list(kernel.inputs) + [o.operand for o in kernel.outputs]
        if any(getattr(o, "view", None) is not None for o in operands):
            return None
    factors: dict = {}
    for p in buffers:
        count = counts.get(p.name)
        if count is None:
            return None
        constant, symbols = P.numel(_count_shape(p))
        if symbols == (r,):
            factors[p.name] = constant
        elif symbols == () and p.role == "in":
            factors[p.name] = None
        else:
            return None
        if count != (P.spell_count((constant, r)) if symbols else P.spell_count((constant,))):
            return None
    if not any(k is not None for k in factors.values()):
        return None
    return f"sym_{r}", factors


def _count_shape(p) -> tuple:
    """The one shape a buffer is read or written with (the first when several agree)."""
    shapes = list(p.read_shapes) + list(p.write_shapes)
    first = tuple(shapes[0])
    if any(P.numel(tuple(s)) != P.numel(first) for s in shapes[1:]):
        return ("?", "?")
    return first


def _tensor_function(fn: P.TensorFunction, src: _Source) -> None:
    launches = []
    any_status = False
    for kernel in fn.kernels:
        if kernel.kind == "map":
            info = _map_kernel(kernel, fn, src)
        elif kernel.kind == "row":
            info = _row_kernel(kernel, fn, src)
        elif kernel.kind == "reduce_all":
            info = _reduce_all_kernel(kernel, fn, src)
        elif kernel.kind == "reduce_cols":
            info = _reduce_cols_kernel(kernel, fn, src)
        elif kernel.kind == "matmul":
            from .gemm import matmul_launch

            info = matmul_launch(kernel, fn, src)
        else:
            raise ValueError(kernel.kind)
        launches.append(info)
        any_status = any_status or info["status"]
    buffers = [p for p in fn.params if p.kind == "buffer"]
    scalars = [p for p in fn.params if p.kind == "scalar"]
    sym = fn.symbol
    # run_<sym>: device pointers in, kernels launched
    run_params = [f"{P.ctype(p.dtype)}* d_{p.name}" for p in buffers]
    run_params += [f"int64_t sym_{b.symbol}" for b in fn.bindings]
    run_params += [f"{P.ctype(p.dtype)} p_{p.name}" for p in scalars]
    R = [f"static int32_t run_{sym}({', '.join(run_params) or 'void'}) {{"]
    R.append("  cudaStream_t stream = (cudaStream_t)ppyb200_stream();")
    R.append("  uint64_t launches = 0;")
    terms = [f"ppyb200_round256({P.spell_count(t.shape)} * (int64_t){P.size_of(t.dtype)})"
             for t in fn.temps]
    terms += [info["scratch"] for info in launches if info.get("scratch")]
    R.append("  ScratchCursor scratch = {nullptr, 0, 0};")
    if terms:
        # temporaries first, then the partials of every reduction, from one arena
        R.append(f"  scratch.size = {' + '.join(terms)};")
        R.append("  scratch.base = (char*)ppyb200_scratch(scratch.size);")
        R.append("  if (scratch.base == nullptr) return PPY_STATUS_RAISED;")
    for t in fn.temps:
        R.append(f"  {P.ctype(t.dtype)}* t_{t.name} = ({P.ctype(t.dtype)}*)ppyb200_scratch_take("
                 f"&scratch, {P.spell_count(t.shape)} * (int64_t){P.size_of(t.dtype)});")
    R.append("  (void)scratch;")
    if any_status:
        R.append("  int32_t* status = ppyb200_status_word();")
        R.append("  if (status == nullptr) return PPY_STATUS_RAISED;")
    else:
        R.append("  int32_t* status = nullptr;")
    for info in launches:
        R.extend("  " + line for line in info["launch"])
    R.append("  ppyb200_count_launches(launches);")
    R.append("  cudaError_t error = cudaGetLastError();")
    R.append(f"  if (error != cudaSuccess) return ppyb200_check((int32_t)error, \"{sym}: launch\");")
    if any_status:
        R.append("  return ppyb200_read_status(status);")
    else:
        R.append("  return PPY_STATUS_OK;")
    R.append("}")
    src.host.append("\n".join(R))
    # bindings and guards, shared by both entry points
    G = []
    for b in fn.bindings:
        const, syms = P.numel(b.divisor)
        divisor = " * ".join([f"(int64_t){const}"] + [f"sym_{s}" for s in syms])
        G.append(f"  int64_t sym_{b.symbol} = 0;")
        G.append("  {")
        G.append(f"    const int64_t divisor = {divisor};")
        G.append("    if (divisor == 0) return PPY_STATUS_FALLBACK;")
        G.append(f"    if ({b.param}_len % divisor != 0) return PPY_STATUS_FALLBACK;")
        G.append(f"    sym_{b.symbol} = {b.param}_len / divisor;")
        G.append("  }")
    for param, shape in fn.guards:
        G.append(f"  if ({param}_len < {P.spell_count(shape)}) return PPY_STATUS_FALLBACK;")
    for symbol, minimum in fn.dim_guards:
        G.append(f"  if (sym_{symbol} < (int64_t){minimum}) return PPY_STATUS_FALLBACK;")
    counts = {}
    for p in buffers:
        shapes = p.read_shapes + p.write_shapes
        if shapes:
            exprs = [P.spell_count(s) for s in shapes]
            counts[p.name] = exprs[0] if len(exprs) == 1 else "ppyb200_max64(" + ", ".join(
                exprs) + ")" if len(exprs) == 2 else exprs[0]
            if len(exprs) > 2:
                acc = exprs[0]
                for e in exprs[1:]:
                    acc = f"ppyb200_max64({acc}, {e})"
                counts[p.name] = acc
    run_args = [f"d_{p.name}" for p in buffers] + [f"sym_{b.symbol}" for b in fn.bindings] + [
        f"p_{p.name}" for p in scalars]
    result_line = f"  if (slot != nullptr) *slot = {fn.result_value};" if fn.result else ""
    # device ABI
    D = [f'extern "C" PPYB200_EXPORT int32_t {sym}__device({", ".join(_abi_params(fn.params) + ["int64_t* slot"])}) {{',
         "  ppyb200_bind_device();"]
    D += G
    for p in buffers:
        D.append(f"  {P.ctype(p.dtype)}* d_{p.name} = {p.name}_ptr;")
    D.append(f"  const int32_t status = run_{sym}({', '.join(run_args)});")
    D.append("  if (status != PPY_STATUS_OK) return status;")
    if result_line:
        D.append(result_line)
    D.append("  return PPY_STATUS_OK;")
    D.append("}")
    src.exports.append("\n".join(D))
    # host ABI
    span = _slices(fn, buffers, counts)
    H = [f'extern "C" PPYB200_EXPORT int32_t {sym}({", ".join(_abi_params(fn.params) + ["int64_t* slot"])}) {{',
         "  ppyb200_bind_device();"]
    H += G
    for p in buffers:
        if p.name not in counts:
            H.append(f"  {P.ctype(p.dtype)}* d_{p.name} = nullptr;")
            continue
        H.append(f"  const int64_t n_{p.name} = {counts[p.name]};")
        H.append(f"  {P.ctype(p.dtype)}* d_{p.name} = ({P.ctype(p.dtype)}*)ppyb200_device_buffer("
                 f"n_{p.name} * (int64_t)sizeof({P.ctype(p.dtype)}));")
    H.append("  int32_t status = PPY_STATUS_OK;")
    conds = [f"(n_{p.name} > 0 && d_{p.name} == nullptr)" for p in buffers if p.name in counts]
    if conds:
        H.append(f"  if ({' || '.join(conds)}) status = PPY_STATUS_RAISED;")
    indent = "  "
    if span is not None:
        # Independent slices along R (a map's elements, a row kernel's rows): large calls go in
        # slices of about PIPELINE_SLICE elements of the widest buffer, over two streams --
        # slice s's copies in, kernel and copies out on stream s % 2 -- so that the copy in of
        # one slice overlaps the kernel and copy out of the one before (host-to-device and
        # device-to-host are separate PCIe directions). Whole operands (per-column vectors) go
        # in first, before the side stream forks from the call's stream.
        sym_n, factors = span
        widest = max(k for k in factors.values() if k is not None)
        rows = max(1, PIPELINE_SLICE // widest)
        slice_args = ([f"d_{p.name} + off * (int64_t){factors[p.name]}"
                       if factors[p.name] is not None else f"d_{p.name}" for p in buffers]
                      + ["len"] + [f"p_{p.name}" for p in scalars])
        H.append(f"  if (status == PPY_STATUS_OK && {sym_n} >= 2 * (int64_t){rows}) {{")
        for p in buffers:
            if factors[p.name] is None:
                H.append(f"    if (status == PPY_STATUS_OK) status = ppyb200_copy_to_device("
                         f"d_{p.name}, {p.name}_ptr, n_{p.name} * (int64_t)sizeof("
                         f"{P.ctype(p.dtype)}));")
        H.append("    void* home = ppyb200_stream();")
        H.append("    void* side = nullptr;")
        H.append("    if (status == PPY_STATUS_OK) status = ppyb200_fork(&side);")
        H.append(f"    for (int64_t off = 0, k = 0; status == PPY_STATUS_OK && off < {sym_n}; "
                 f"off += {rows}, ++k) {{")
        H.append(f"      const int64_t len = {sym_n} - off < (int64_t){rows} ? "
                 f"{sym_n} - off : (int64_t){rows};")
        H.append("      ppyb200_set_stream(k % 2 ? side : home);")
        for p in buffers:
            k = factors[p.name]
            if k is not None and p.role in ("in", "inout"):
                H.append(f"      if (status == PPY_STATUS_OK) status = ppyb200_copy_to_device("
                         f"d_{p.name} + off * (int64_t){k}, {p.name}_ptr + off * (int64_t){k}, "
                         f"len * (int64_t){k} * (int64_t)sizeof({P.ctype(p.dtype)}));")
        H.append(f"      if (status == PPY_STATUS_OK) status = run_{sym}({', '.join(slice_args)});")
        for p in buffers:
            k = factors[p.name]
            if k is not None and p.role in ("out", "inout"):
                H.append(f"      if (status == PPY_STATUS_OK) status = ppyb200_copy_to_host("
                         f"{p.name}_ptr + off * (int64_t){k}, d_{p.name} + off * (int64_t){k}, "
                         f"len * (int64_t){k} * (int64_t)sizeof({P.ctype(p.dtype)}));")
        H.append("    }")
        H.append("    ppyb200_set_stream(home);")
        H.append("    if (side != nullptr) { const int32_t joined = ppyb200_join(side); "
                 "if (status == PPY_STATUS_OK) status = joined; }")
        H.append("  } else {")
        indent = "    "
    for p in buffers:
        if p.name in counts and p.role in ("in", "inout"):
            H.append(f"{indent}if (status == PPY_STATUS_OK) status = ppyb200_copy_to_device(d_{p.name}, "
                     f"{p.name}_ptr, n_{p.name} * (int64_t)sizeof({P.ctype(p.dtype)}));")
    H.append(f"{indent}if (status == PPY_STATUS_OK) status = run_{sym}({', '.join(run_args)});")
    for p in buffers:
        if p.name in counts and p.role in ("out", "inout"):
            H.append(f"{indent}if (status == PPY_STATUS_OK) status = ppyb200_copy_to_host({p.name}_ptr, "
                     f"d_{p.name}, n_{p.name} * (int64_t)sizeof({P.ctype(p.dtype)}));")
    if span is not None:
        H.append("  }")
    H.append("  { const int32_t synced = ppyb200_sync(); if (status == PPY_STATUS_OK) status = synced; }")
    for p in buffers:
        if p.name in counts:
            H.append(f"  ppyb200_release_buffer(d_{p.name});")
    H.append("  if (status != PPY_STATUS_OK) return status;")
    if result_line:
        H.append(result_line)
    H.append("  return PPY_STATUS_OK;")
    H.append("}")
    src.exports.append("\n".join(H))


# -- scalar functions and parallel kernels -------------------------------------------------


#: Consecutive indices a thread hands a parallel.for/reduce body in one call. The body loops
#: over its own [begin, end) (lower_parallel.py:141-318 gives it that shape), so a lane runs
#: the whole run before the warp reconverges at the call's return: one index per call made
#: every index cost the warp its longest lane's work (Collatz: path lengths differ by 10x).
PARALLEL_RUN = 1


def _parallel_kernel(k: ParallelKernel, src: _Source) -> None:
    caps = [f"{t} {n}" for t, n in k.captures]
    cap_names = [n for _, n in k.captures]
    T = THREADS
    if k.kind == "reduce":
        rt = P.ctype(k.result)
        op = _COMBINE[k.reduce]
        ident = identity_literal(k.reduce, k.result)
        L = [f"static __global__ void __launch_bounds__({T}) {k.name}_part("
             + ", ".join(caps + ["int64_t begin", "int64_t end", f"{rt} start",
                                 f"{rt}* __restrict__ partials", "int32_t* status"]) + ") {",
             f"  {rt} acc = start;",
             f"  const int64_t runs = (end - begin + {PARALLEL_RUN} - 1) / {PARALLEL_RUN};",
             "  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < runs; "
             "t += (int64_t)gridDim.x * blockDim.x) {",
             f"    const int64_t i = begin + t * {PARALLEL_RUN};",
             f"    const int64_t stop = end - i < {PARALLEL_RUN} ? end : i + {PARALLEL_RUN};",
             f"    {rt} next;",
             f"    const int32_t s = {k.body}(" + ", ".join(cap_names + ["i", "stop", "acc", "&next"]) + ");",
             "    if (s != PPY_STATUS_OK) {",
             "      ppyb200::raise_status(status, s);",
             "      break;",
             "    }",
             "    acc = next;",
             "  }"]
        L += _block_reduce_lines(rt, op, "acc")
        L.append("  if (threadIdx.x == 0) partials[blockIdx.x] = acc;")
        L.append("}")
        L2 = [f"static __global__ void __launch_bounds__({T}) {k.name}_fin(const {rt}* __restrict__ partials, "
              f"int64_t parts, {rt} init, {rt}* __restrict__ out) {{",
              f"  {rt} acc = {ident};",
              f"  for (int64_t i = threadIdx.x; i < parts; i += blockDim.x) acc = {op}::apply(acc, partials[i]);"]
        L2 += _block_reduce_lines(rt, op, "acc")
        L2.append(f"  if (threadIdx.x == 0) out[0] = {op}::apply(init, acc);")
        L2.append("}")
        src.kernels.append("\n".join(L))
        src.kernels.append("\n".join(L2))
        # start value of every thread: the op's identity (add/mul) or init (min/max),
        # as parallel.identity has it (ir/dialects/parallel.py:666-673)
        start = ident if k.reduce in ("add", "mul") else "init"
        H = [f"static int32_t launch_{k.name}(" + ", ".join(caps + ["int64_t begin", "int64_t end",
                                                                  f"{rt} init", f"{rt}* result"]) + ") {",
             "  cudaStream_t stream = (cudaStream_t)ppyb200_stream();",
             "  if (end <= begin) { *result = init; return PPY_STATUS_OK; }",
             f"  const int64_t parts = ppyb200_parallel_blocks((end - begin + {PARALLEL_RUN} - 1) / "
             f"{PARALLEL_RUN}, {T});",
             f"  {rt}* part = ({rt}*)ppyb200_scratch((parts + 1) * (int64_t)sizeof({rt}));",
             "  if (part == nullptr) return PPY_STATUS_RAISED;",
             "  int32_t* status = ppyb200_status_word();",
             "  if (status == nullptr) return PPY_STATUS_RAISED;",
             f"  {k.name}_part<<<(unsigned)parts, {T}, 0, stream>>>(" + ", ".join(
                 cap_names + ["begin", "end", start, "part", "status"]) + ");",
             f"  {k.name}_fin<<<1, {T}, 0, stream>>>(part, parts, init, part + parts);",
             "  ppyb200_count_launches(2);",
             "  cudaError_t error = cudaGetLastError();",
             f"  if (error != cudaSuccess) return ppyb200_check((int32_t)error, \"{k.name}\");",
             f"  int32_t s = ppyb200_copy_to_host(result, part + parts, sizeof({rt}));",
             "  if (s != PPY_STATUS_OK) return s;",
             "  return ppyb200_read_status(status);",
             "}"]
        src.host.append("\n".join(H))
        return
    if k.kind == "for":
        L = [f"static __global__ void __launch_bounds__({T}) {k.name}_k("
             + ", ".join(caps + ["int64_t begin", "int64_t end", "int32_t* status"]) + ") {",
             f"  const int64_t runs = (end - begin + {PARALLEL_RUN} - 1) / {PARALLEL_RUN};",
             "  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < runs; "
             "t += (int64_t)gridDim.x * blockDim.x) {",
             f"    const int64_t i = begin + t * {PARALLEL_RUN};",
             f"    const int64_t stop = end - i < {PARALLEL_RUN} ? end : i + {PARALLEL_RUN};",
             f"    const int32_t s = {k.body}(" + ", ".join(cap_names + ["i", "stop"]) + ");",
             "    if (s != PPY_STATUS_OK) {",
             "      ppyb200::raise_status(status, s);", "      break;", "    }", "  }", "}"]
        extra_params, extra_args = [], []
    else:  # map
        ot = P.ctype(k.out_dtype)
        L = [f"static __global__ void __launch_bounds__({T}) {k.name}_k("
             + ", ".join(caps + ["int64_t begin", "int64_t end", f"{ot}* out", "int32_t* status"]) + ") {",
             "  const int64_t count = end - begin;",
             "  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < count; "
             "t += (int64_t)gridDim.x * blockDim.x) {",
             "    const int64_t i = begin + t;",
             f"    {ot} value;",
             f"    const int32_t s = {k.body}(" + ", ".join(cap_names + ["i", "&value"]) + ");",
             "    if (s != PPY_STATUS_OK) {",
             "      ppyb200::raise_status(status, s);", "      break;", "    }",
             "    out[i] = value;", "  }", "}"]
        extra_params, extra_args = [f"{ot}* out"], ["out"]
    src.kernels.append("\n".join(L))
    H = [f"static int32_t launch_{k.name}(" + ", ".join(caps + ["int64_t begin", "int64_t end"] + extra_params) + ") {",
         "  cudaStream_t stream = (cudaStream_t)ppyb200_stream();",
         "  if (end <= begin) return PPY_STATUS_OK;",
         "  int32_t* status = ppyb200_status_word();",
         "  if (status == nullptr) return PPY_STATUS_RAISED;",
         ("  const int64_t blocks = ppyb200_parallel_blocks("
          + (f"(end - begin + {PARALLEL_RUN} - 1) / {PARALLEL_RUN}" if k.kind == "for"
             else "end - begin") + f", {T});"),
         f"  {k.name}_k<<<(unsigned)blocks, {T}, 0, stream>>>(" + ", ".join(
             cap_names + ["begin", "end"] + extra_args + ["status"]) + ");",
         "  ppyb200_count_launches(1);",
         "  cudaError_t error = cudaGetLastError();",
         f"  if (error != cudaSuccess) return ppyb200_check((int32_t)error, \"{k.name}\");",
         "  return ppyb200_read_status(status);",
         "}"]
    src.host.append("\n".join(H))


def _scalar_function(fn: P.ScalarFunction, src: _Source) -> None:
    src.host.append(fn.host_source)
    atoms = _abi_params(fn.params)
    call = []
    for p in fn.params:
        if p.kind == "buffer":
            call += [f"{p.name}_ptr", f"{p.name}_len"]
        elif p.kind == "ptr":
            call.append(p.name)
        else:
            call.append(f"p_{p.name}")
    result_t = P.ctype(fn.result) if fn.result else None
    for suffix in ("", "__device"):
        E = [f'extern "C" PPYB200_EXPORT int32_t {fn.symbol}{suffix}({", ".join(atoms + ["int64_t* slot"])}) {{',
             "  ppyb200_bind_device();"]
        if result_t:
            E.append(f"  {result_t} result{{}};")
            E.append(f"  const int32_t status = host_{fn.name}({', '.join(call + ['&result'])});")
            E.append("  if (status == PPY_STATUS_OK && slot != nullptr) *slot = (int64_t)result;")
        else:
            E.append(f"  const int32_t status = host_{fn.name}({', '.join(call)});")
        E.append("  return status;")
        E.append("}")
        src.exports.append("\n".join(E))


PRELUDE = r'''// Generated by the PPy b200 backend from module @{module}. Do not edit: regenerate
// with `ppy build --backend b200`.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include "ppyb200_device.cuh"
#include "ppyb200.h"

// Only the entry points leave the library: kernels and helpers have internal linkage,
// so modules loaded side by side never call each other's code.
#define PPYB200_EXPORT __attribute__((visibility("default")))

// This library's CUDA runtime follows the device the calling thread bound with
// ppyb200_init (each library carries its own runtime; the context is shared).
static inline void ppyb200_bind_device(void) {
  static thread_local int bound = -2;
  const int want = ppyb200_current_device();
  if (want >= 0 && want != bound) {
    cudaSetDevice(want);
    bound = want;
  }
}
static inline bool ppyb200_aligned(const void* p, int64_t bytes) {
  return ((uintptr_t)p % (uintptr_t)bytes) == 0;
}
static inline int64_t ppyb200_max64(int64_t a, int64_t b) { return a > b ? a : b; }
static inline int64_t ppyb200_round256(int64_t b) { return (b + 255) / 256 * 256; }
// Grid sizes in whole waves of the device's SMs (148 on a B200).
static inline int64_t ppyb200_blocks(int64_t work, int64_t per_block) {
  int64_t blocks = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 64;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : blocks;
}
static inline int64_t ppyb200_row_blocks(int64_t rows, int64_t rows_per_block) {
  int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 32;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : blocks;
}
static inline int64_t ppyb200_reduce_blocks(int64_t n, int64_t threads) {
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : blocks;
}
static inline int64_t ppyb200_col_chunks(int64_t rows, int64_t col_blocks) {
  int64_t want = ((int64_t)ppyb200_sm_count() * 8 + col_blocks - 1) / col_blocks;
  if (want > rows) want = rows;
  if (want > 65535) want = 65535;
  return want < 1 ? 1 : want;
}
static inline int64_t ppyb200_parallel_blocks(int64_t n, int64_t threads) {
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : blocks;
}
// One call's temporaries and reduction partials, carved from the stream's scratch arena.
struct ScratchCursor {
  char* base;
  int64_t size;
  int64_t at;
};
static inline void* ppyb200_scratch_take(ScratchCursor* s, int64_t bytes) {
  if (s->at + bytes > s->size) {
    ppyb200_set_error("scratch arena exhausted");
    return nullptr;
  }
  void* p = s->base + s->at;
  s->at += ppyb200_round256(bytes);
  return p;
}
'''


def module_source(plan: P.ModulePlan, device_sources: list[str], kernels: list) -> str:
    """The CUDA C++ translation unit of one planned module."""
    src = _Source()
    for fn in plan.functions:
        if fn.kind == "tensor":
            _tensor_function(fn, src)
    for k in kernels:
        _parallel_kernel(k, src)
    scalar_fns = [fn for fn in plan.functions if fn.kind == "scalar"]
    prototypes = []
    for text in device_sources:
        prototypes.append(text.split(" {", 1)[0] + ";")
    host_protos = [fn.host_source.split(" {", 1)[0] + ";" for fn in scalar_fns]
    for fn in scalar_fns:
        _scalar_function(fn, src)
    parts = [PRELUDE.replace("{module}", plan.name)]
    if any(k.kind == "matmul" for fn in plan.functions if fn.kind == "tensor" for k in fn.kernels):
        parts.append('#include "gemm_sm100.cuh"\n#include "gemm_simt.cuh"\n#include "gemm_f32.cuh"')
    parts += prototypes
    parts += device_sources
    parts += src.kernels
    parts += host_protos
    parts += src.host
    parts += src.exports
    return "\n\n".join(parts) + "\n"
