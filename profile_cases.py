"""Single-kernel cases for Nsight Compute: each runs one hand-written kernel a few times on
seeded inputs of the benchmark's shapes, so `ncu -k <kernel> -s <warm-up> -c 1` can capture
one launch of it alone.

    python profile_cases.py gemm        # matmul_bf16_pair_kernel, 8192^3, K-major B
    python profile_cases.py attention   # causal_kernel, batch 32 x 1024, 12 heads
    python profile_cases.py fc          # matmul_bf16_pair_kernel, GELU epilogue,
                                                 # GPT-2 FC (32768 x 3072 x 768)
    python profile_cases.py proj        # matmul_bf16_pair_kernel, residual quads epilogue,
                                         # GPT-2 proj (32768 x 768 x 3072, x += f W^T + b)
    python profile_cases.py gemm_f32    # matmul_tf32x3_pair_kernel, f32 4096^3 (after the
                                         # two split kernels of each call)
    python profile_cases.py lm_head     # matmul_bf16_pair_kernel, quads epilogue,
                                                 # 50257 logits a row in rows 50272 apart

Each case launches its kernel three times (two warm-ups, then the one to capture: `-s 2`).
The GEMM cases run CTA pairs, the default from 256 rows; `ppyb200_set_gemm_form` pins one CTA
per tile for a capture of `matmul_bf16_kernel`.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))


def main() -> None:
    import torch

    from ppy_b200 import gpt2, runtime

    parser = argparse.ArgumentParser()
    parser.add_argument("case", choices=["gemm", "gemm_f32", "attention", "fc", "proj",
                                         "lm_head"])
    case = parser.parse_args().case
    runtime.init(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    runtime.set_stream(stream)
    lib = runtime.library()
    gpt2._bind(lib)
    g = torch.Generator(device="cuda").manual_seed(0)

    def rand(*shape, dtype=torch.bfloat16):
        return torch.randn(*shape, device="cuda", generator=g).to(dtype)

    for _ in range(3):
        if case in ("gemm", "lm_head"):
            if not hasattr(main, "operands"):
                m, n, k = (8192, 8192, 8192) if case == "gemm" else (4096, 50257, 768)
                ldc = n if case == "gemm" else 50272  # the GPT-2 forward's logits rows
                main.operands = (rand(m, k), rand(n, k), torch.empty(m, ldc, device="cuda"),
                                 ldc, m, n, k)
            a, bt, c, ldc, m, n, k = main.operands
            status = lib.ppyb200_matmul_bf16_kmajor_ld(a.data_ptr(), bt.data_ptr(), None,
                                                       c.data_ptr(), ldc, m, n, k)
        elif case == "gemm_f32":
            if not hasattr(main, "operands"):
                import ctypes

                lib.ppyb200_matmul_f32.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
                main.operands = tuple(rand(4096, 4096, dtype=torch.float32) for _ in range(2)) + (
                    torch.empty(4096, 4096, device="cuda"),)
            a, b, c = main.operands
            status = lib.ppyb200_matmul_f32(a.data_ptr(), b.data_ptr(), None, c.data_ptr(),
                                            4096, 4096, 4096)
        elif case == "proj":
            if not hasattr(main, "operands"):
                main.operands = (rand(32768, 3072), rand(768, 3072),
                                 torch.zeros(768, device="cuda"),
                                 torch.zeros(32768, 768, device="cuda"))
            f, w, b, x = main.operands
            status = lib.ppyb200_linear_residual(f.data_ptr(), w.data_ptr(), b.data_ptr(),
                                                 x.data_ptr(), 32768, 768, 3072, None)
        elif case == "attention":
            if not hasattr(main, "operands"):
                main.operands = (rand(32 * 1024, 3 * 768), rand(32 * 12 * 64, 1024),
                                 torch.empty(32 * 1024, 768, device="cuda", dtype=torch.bfloat16))
            qkv, vt, out = main.operands
            status = lib.ppyb200_attention_causal_vt_bf16(qkv.data_ptr(), vt.data_ptr(),
                                                          out.data_ptr(), 32, 1024, 12, 64, None)
        else:
            if not hasattr(main, "operands"):
                main.operands = (rand(32768, 768), rand(3072, 768),
                                 torch.zeros(3072, device="cuda"),
                                 torch.empty(32768, 3072, device="cuda", dtype=torch.bfloat16))
            h, w, b, f = main.operands
            status = lib.ppyb200_linear_bf16(h.data_ptr(), w.data_ptr(), b.data_ptr(),
                                             f.data_ptr(), 32768, 3072, 768, 1, None)
        if status != 0:
            raise SystemExit(f"{case}: {runtime.last_error()}")
    torch.cuda.synchronize()
    print(f"{case}: ok")


if __name__ == "__main__":
    main()
