"""The kernel plan: what the b200 backend makes of one IR function.

`translate` (which reads PPy's canonical IR) produces these objects and `codegen`
(which knows nothing of PPy) turns them into CUDA C++. A plan is plain data:
shapes are tuples of ints and symbol names, scalar programs are lists of SSA
statements, and every tensor a kernel touches is an `Operand` naming where its
memory is (a buffer parameter or a temporary) and its row-major shape.
"""

from __future__ import annotations

from dataclasses import dataclass, field

#: Element types the backend takes, with their C++ spelling and size in bytes.
CTYPES = {
    "f32": ("float", 4),
    "f64": ("double", 8),
    "bf16": ("__nv_bfloat16", 2),
    "i64": ("int64_t", 8),
    "i32": ("int32_t", 4),
    "i16": ("int16_t", 2),
    "i8": ("int8_t", 1),
    "u64": ("uint64_t", 8),
    "u32": ("uint32_t", 4),
    "u16": ("uint16_t", 2),
    "u8": ("uint8_t", 1),
    "bool": ("bool", 1),
    "index": ("int64_t", 8),
}

FLOATS = frozenset({"f32", "f64", "bf16"})

Dim = "int | str"


def ctype(dtype: str) -> str:
    return CTYPES[dtype][0]


def size_of(dtype: str) -> int:
    return CTYPES[dtype][1]


def is_float(dtype: str) -> bool:
    return dtype in FLOATS


def numel(shape: tuple) -> tuple[int, tuple[str, ...]]:
    """A shape's element count as (constant factor, symbol factors)."""
    constant = 1
    symbols: list[str] = []
    for dim in shape:
        if isinstance(dim, int):
            constant *= dim
        else:
            symbols.append(dim)
    return constant, tuple(symbols)


def spell_count(shape: tuple) -> str:
    """C++ expression (int64_t) for a shape's element count; symbols are locals."""
    constant, symbols = numel(shape)
    parts = [f"(int64_t){constant}"] + [f"sym_{s}" for s in symbols]
    return " * ".join(parts)


def spell_dims(shape: tuple) -> list[str]:
    return [f"(int64_t){d}" if isinstance(d, int) else f"sym_{d}" for d in shape]


# -- index arithmetic of strided views: ints where known, C++ int64_t expressions otherwise ----


def dim_term(dim):
    """A dimension as an index term: an int, or the bound symbol's local."""
    return dim if isinstance(dim, int) else f"sym_{dim}"


def spell_term(x) -> str:
    return f"(int64_t){x}" if isinstance(x, int) else x


def term_mul(a, b):
    if isinstance(a, int) and isinstance(b, int):
        return a * b
    if a == 0 or b == 0:
        return 0
    if a == 1:
        return b
    if b == 1:
        return a
    return f"({spell_term(a)} * {spell_term(b)})"


def term_add(a, b):
    if isinstance(a, int) and isinstance(b, int):
        return a + b
    if a == 0:
        return b
    if b == 0:
        return a
    return f"({spell_term(a)} + {spell_term(b)})"


def contiguous_strides(shape: tuple) -> tuple:
    """Row-major element strides of `shape` (lower_tensor's `shapes.strides_of`)."""
    strides = [1] * len(shape)
    running = 1
    for axis in reversed(range(len(shape))):
        strides[axis] = running
        running = term_mul(running, dim_term(shape[axis]))
    return tuple(strides)


@dataclass
class Param:
    """One IR function parameter and the ABI atoms it becomes."""

    name: str
    kind: str  # "buffer" | "scalar" | "ptr"
    dtype: str
    #: For buffers: "in" (read), "out" (written), "inout", or "" (unused).
    role: str = ""
    #: Elements of the buffer the function reads and writes (shapes whose counts bound it).
    read_shapes: list = field(default_factory=list)
    write_shapes: list = field(default_factory=list)


@dataclass
class Operand:
    """A tensor in memory: a buffer parameter (`param`) or a temporary (`temp`).

    With `view` = (offset, strides) the tensor is a strided view of that memory (the
    reference's `_View`, lower_tensor.py:695-714): element (i0, i1, ...) of `shape` sits at
    offset + i0 * strides[0] + i1 * strides[1] + ..., offset and strides in elements, each an
    int or a C++ expression over the bound symbols; without it the tensor is contiguous and
    row-major."""

    source: str  # "param" | "temp"
    name: str
    dtype: str
    shape: tuple
    view: tuple | None = None

    @property
    def pointer(self) -> str:
        return f"d_{self.name}" if self.source == "param" else f"t_{self.name}"


@dataclass
class Stmt:
    """One scalar SSA statement of a kernel's element program.

    `op` is one of: input (args = (operand index,)), const (attrs value), param
    (attrs name), add, sub, mul, div, mod, neg, and, or, xor, shl, shr, cmp (attrs
    predicate), select, cast, math (attrs fn), pow, special (attrs fn), reduce
    (attrs kind; ROW kernels only).
    """

    var: str
    op: str
    args: tuple = ()
    dtype: str = "f32"
    attrs: dict = field(default_factory=dict)


@dataclass
class Output:
    var: str
    operand: Operand


@dataclass
class MapKernel:
    """One element of every output from one element of each input, over `shape`."""

    name: str
    shape: tuple
    inputs: list
    program: list
    outputs: list
    kind: str = "map"


@dataclass
class RowKernel:
    """A group over rows: the leading axes of `shape` are rows, the trailing `reduced`
    axes (static, `cols` elements) are one row; reductions fold a row to a scalar.
    Inputs are full elements, per-row scalars, per-column vectors, or scalars."""

    name: str
    shape: tuple
    reduced: int
    cols: int
    inputs: list
    program: list
    outputs: list
    kind: str = "row"


@dataclass
class ReduceAllKernel:
    """A fold of a whole element stream (`program` yields `var`) to one value."""

    name: str
    shape: tuple
    inputs: list
    program: list
    var: str
    reduce: str
    dtype: str
    output: Operand
    kind: str = "reduce_all"


@dataclass
class ReduceColsKernel:
    """A fold over the leading `reduced` axes of `shape`: one value per column."""

    name: str
    shape: tuple
    reduced: int
    inputs: list
    program: list
    var: str
    reduce: str
    dtype: str
    output: Operand
    kind: str = "reduce_cols"


@dataclass
class MatmulKernel:
    """C = A @ B (+ an elementwise epilogue over [M, N]); bf16 or f32 operands, f32 result."""

    name: str
    a: Operand
    b: Operand
    m: object
    n: int
    k: int
    #: The epilogue's program: input 0 is the product's element; other inputs follow.
    inputs: list
    program: list
    outputs: list
    kind: str = "matmul"


@dataclass
class Binding:
    """`symbol` = len(param) / divisor (the reference's `bind_symbols`)."""

    symbol: str
    param: str
    divisor: tuple  # a shape whose element count divides the length


@dataclass
class Temp:
    name: str
    dtype: str
    shape: tuple


@dataclass
class TensorFunction:
    name: str
    symbol: str
    params: list
    result: str | None
    result_value: int
    bindings: list
    #: (param, shape): guard `len(param) >= numel(shape)`, in IR order.
    guards: list
    temps: list
    kernels: list
    kind: str = "tensor"
    #: (symbol, minimum): guard `symbol >= minimum` (a slice that stops inside a symbolic
    #: dimension).
    dim_guards: list = field(default_factory=list)


@dataclass
class ScalarFunction:
    """A function of core arithmetic and control flow, possibly launching parallel
    loops; its C++ body is emitted directly from the IR."""

    name: str
    symbol: str
    params: list
    result: str | None
    host_source: str
    device_sources: list
    kernels: list
    kind: str = "scalar"


@dataclass
class ModulePlan:
    name: str
    functions: list
    notes: list = field(default_factory=list)
    #: Device copies of the functions parallel bodies run, and the parallel kernels.
    device_sources: list = field(default_factory=list)
    parallel_kernels: list = field(default_factory=list)
