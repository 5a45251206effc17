"""Matmul kernels of a plan: `tensor.matmul` / `linalg.matmul` with the elementwise group
that follows it (the bias add FuseTensor leaves) fused into the epilogue.

bf16 operands with K a multiple of 64 run on the tcgen05 kernel (csrc/gemm_sm100.cuh)
after B, row-major [K, N] as the IR has it, is transposed into the scratch arena; f32
operands run on the same kernel as three tf32 products after a split pass into the arena
(csrc/gemm_f32.cuh); every other case runs on the CUDA-core kernel (csrc/gemm_simt.cuh). The epilogue is a functor
generated from the group's element program: input 0 is the product's element, the other
inputs are read per row, per column, per element or once.
"""

from __future__ import annotations

from . import plan as P
from .codegen import _compute_dtype, _scalar_params, presence, stmt_expr
from .scalar_c import Unsupported

__all__ = ["matmul_launch"]


def _classes(kernel: P.MatmulKernel) -> list[str]:
    frame = (kernel.m, kernel.n)
    out = []
    for i, operand in enumerate(kernel.inputs):
        if i == 0:
            out.append("acc")
            continue
        flags = presence(operand.shape, frame)
        out.append({(True, True): "elem", (True, False): "rows", (False, True): "cols",
                    (False, False): "scalar"}[tuple(flags)])
    return out


def matmul_launch(kernel: P.MatmulKernel, fn: P.TensorFunction, src) -> dict:
    params_by_name = {p.name: p for p in fn.params}
    if len(kernel.outputs) != 1:
        raise Unsupported("a matmul whose product and epilogue are both stored",
                          "one stored result per matmul")
    out = kernel.outputs[0]
    if out.operand.dtype not in ("f32", "bf16", "f64"):
        raise Unsupported(f"a matmul stored as {out.operand.dtype}", "float matmul results")
    classes = _classes(kernel)
    dtypes = {s.var: s.dtype for s in kernel.program}
    scalars = _scalar_params(kernel.program, params_by_name)
    name = kernel.name
    # --- epilogue functor
    members = []
    for i, operand in enumerate(kernel.inputs[1:], start=1):
        members.append(f"const {P.ctype(operand.dtype)}* __restrict__ in{i};")
    members += [f"{P.ctype(t)} p_{n};" for n, t in scalars]
    body = []
    for s in kernel.program:
        ct = P.ctype(_compute_dtype(s.dtype))
        if s.op == "input":
            i = s.args[0]
            c = classes[i]
            if c == "acc":
                e = "acc"
            else:
                idx = {"elem": "row * n + col", "rows": "row", "cols": "col", "scalar": "0"}[c]
                e = f"__ldg(in{i} + {idx})"
                if kernel.inputs[i].dtype == "bf16":
                    e = f"ppyb200::convert<float, __nv_bfloat16>({e})"
            body.append(f"    const {ct} {s.var} = {e};")
            continue
        expr, pre = stmt_expr(s, lambda v: v, dtypes)
        body.extend("    " + p for p in pre)
        body.append(f"    const {ct} {s.var} = {expr};")
    result_ct = P.ctype(_compute_dtype(dtypes[out.var]))
    out_ct = P.ctype(out.operand.dtype)
    functor = [f"struct {name}_epi {{"] + ["  " + m for m in members] + [
        "  int64_t n;",
        "  int32_t* status;",
        f"  {out_ct}* __restrict__ out;",
        "  __device__ __forceinline__ void store(float acc, int64_t row, int64_t col) const {"
        ] + body + [
        f"    out[row * n + col] = ppyb200::convert<{out_ct}, {result_ct}>({out.var});",
        "  }",
        "  __device__ __forceinline__ void store_column(const float (&acc)[32], int64_t row0, "
        "int64_t col, int64_t rows) const {",
        "    ppyb200::gemm::for_column(*this, acc, row0, col, rows);",
        "  }", "};"]
    src.kernels.append("\n".join(functor))
    # --- launch
    a, b = kernel.a, kernel.b
    m_expr = P.spell_count((kernel.m,))
    init = ", ".join([o.pointer for o in kernel.inputs[1:]] + [f"p_{n}" for n, _ in scalars]
                     + ["n", "status", out.operand.pointer])
    ct = P.ctype(a.dtype)
    lines = ["{",
             f"  const int64_t m = {m_expr}, n = {kernel.n}, k = {kernel.k};",
             f"  {name}_epi epi{{{init}}};",
             "  if (m > 0) {"]
    tensor_cores = a.dtype == "bf16" and kernel.k % 64 == 0
    tf32x3 = a.dtype == "f32" and b.dtype == "f32"
    if tf32x3:
        lines += [
            "    // f32 operands: three tf32 products on the tensor cores (gemm_f32.cuh); the",
            "    // split operands and the non-finite flag live in the scratch arena",
            "    float* work = (float*)ppyb200_scratch_take(&scratch, ppyb200::gemm::tf32x3_work_bytes(m, n, k));",
            "    if (work == nullptr) return PPY_STATUS_RAISED;",
            f"    cudaError_t e = ppyb200::gemm::launch_tf32x3((const float*){a.pointer}, (const float*){b.pointer}, "
            "work, m, n, k, epi, status, ppyb200_sm_count(), stream);",
            f"    if (e != cudaSuccess) return ppyb200_check((int32_t)e, \"{name}\");",
            "    launches += 4;"]
    elif tensor_cores:
        lines += [
            f"    if (ppyb200_aligned({a.pointer}, 16) && m < (1ll << 31)) {{",
            "      // B is row-major [K, N]; the tensor-core kernel reads it K-major [N, K]",
            "      __nv_bfloat16* bt = (__nv_bfloat16*)ppyb200_scratch_take(&scratch, n * k * 2);",
            "      if (bt == nullptr) return PPY_STATUS_RAISED;",
            f"      cudaError_t e = ppyb200::launch_transpose((const __nv_bfloat16*){b.pointer}, bt, k, n, stream);",
            "      if (e == cudaSuccess) e = ppyb200::gemm::launch("
            f"(const __nv_bfloat16*){a.pointer}, bt, m, n, k, epi, status, ppyb200_sm_count(), stream);",
            f"      if (e != cudaSuccess) return ppyb200_check((int32_t)e, \"{name}\");",
            "      launches += 2;",
            "    } else {",
            f"      cudaError_t e = ppyb200::simt::launch(({'const ' + ct}*){a.pointer}, ({'const ' + ct}*){b.pointer}, m, n, k, epi, stream);",
            f"      if (e != cudaSuccess) return ppyb200_check((int32_t)e, \"{name}\");",
            "      launches += 1;",
            "    }"]
    else:
        lines += [
            f"    cudaError_t e = ppyb200::simt::launch(({'const ' + ct}*){a.pointer}, ({'const ' + ct}*){b.pointer}, m, n, k, epi, stream);",
            f"    if (e != cudaSuccess) return ppyb200_check((int32_t)e, \"{name}\");",
            "    launches += 1;"]
    lines += ["  }", "}"]
    info = {"launch": lines, "status": tensor_cores or tf32x3, "gemm": True}
    if tensor_cores:
        info["scratch"] = f"ppyb200_round256((int64_t){kernel.n} * {kernel.k} * 2)"
    elif tf32x3:
        info["scratch"] = (f"ppyb200::gemm::tf32x3_work_bytes({m_expr}, (int64_t){kernel.n}, "
                           f"(int64_t){kernel.k})")
    return info
