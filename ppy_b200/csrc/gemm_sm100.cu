// The C-ABI matmul entry points of libppyb200 (include/ppyb200.h): bf16 x bf16 -> f32 with
// an optional f32 bias row, on tcgen05 tensor cores for whole 128x256x64 tiles and on the
// CUDA cores otherwise.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/ppyb200.h"
#include "gemm_sm100.cuh"
#include "gemm_simt.cuh"

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int32_t g_gemm_form = PPYB200_GEMM_BY_SHAPE;

int32_t finish(cudaError_t error, const char* what, uint64_t launched) {
  if (error != cudaSuccess) return ppyb200_check((int32_t)error, what);
  ppyb200_count_launches(launched);
  return PPYB200_OK;
}

}  // namespace

extern "C" {

int32_t ppyb200_set_gemm_form(int32_t form) {
  if (form != PPYB200_GEMM_BY_SHAPE && form != PPYB200_GEMM_PAIRS &&
      form != PPYB200_GEMM_SINGLE) {
    ppyb200_set_error("ppyb200_set_gemm_form: 0 (by shape), 1 (CTA pairs) or 2 (one CTA)");
    return PPYB200_RAISED;
  }
  const int32_t before = g_gemm_form;
  g_gemm_form = form;
  return before;
}

int32_t ppyb200_gemm_form(void) { return g_gemm_form; }

int32_t ppyb200_transpose_bf16(const uint16_t* b, uint16_t* bt, int64_t k, int64_t n) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  cudaError_t e = ppyb200::launch_transpose(reinterpret_cast<const __nv_bfloat16*>(b),
                                            reinterpret_cast<__nv_bfloat16*>(bt), k, n, stream);
  return finish(e, "ppyb200_transpose_bf16", 1);
}

int32_t ppyb200_matmul_bf16_kmajor(const uint16_t* a, const uint16_t* bt, const float* bias,
                                   float* c, int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) {
    ppyb200_set_error("ppyb200_matmul_bf16_kmajor: negative extent");
    return PPYB200_RAISED;
  }
  if (m == 0 || n == 0) return PPYB200_OK;
  if (!ppyb200::gemm::tileable(m, n, k) || !aligned16(a) || !aligned16(bt)) {
    ppyb200_set_error("ppyb200_matmul_bf16_kmajor: K % 64 and 16-byte aligned operands are "
                      "required");
    return PPYB200_FALLBACK;
  }
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  int32_t* status = ppyb200_status_word();
  if (status == nullptr) return PPYB200_RAISED;
  // C = A.B + bias by columns of 32 rows (measured faster here than the four-column form
  // whenever the rows allow either: 0.80 against 0.85 ms at 8192^3)
  cudaError_t e = ppyb200::gemm::launch(reinterpret_cast<const __nv_bfloat16*>(a),
                                        reinterpret_cast<const __nv_bfloat16*>(bt), m, n, k,
                                        ppyb200::gemm::BiasEpilogue{bias, c, n}, status,
                                        ppyb200_sm_count(), stream);
  return finish(e, "ppyb200_matmul_bf16_kmajor", 1);
}

int32_t ppyb200_matmul_bf16(const uint16_t* a, const uint16_t* b, const float* bias, float* c,
                            int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) {
    ppyb200_set_error("ppyb200_matmul_bf16: negative extent");
    return PPYB200_RAISED;
  }
  if (m == 0 || n == 0) return PPYB200_OK;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(a);
  const auto* B = reinterpret_cast<const __nv_bfloat16*>(b);
  if (!ppyb200::gemm::tileable(m, n, k) || !aligned16(a)) {
    ppyb200::gemm::BiasEpilogue epi{bias, c, n};
    cudaError_t e = ppyb200::simt::launch(A, B, m, n, k, epi, stream);
    return finish(e, "ppyb200_matmul_bf16 (CUDA cores)", 1);
  }
  // B arrives row-major [K, N]; the tensor-core kernel reads it K-major ([N, K]).
  void* bt = ppyb200_scratch(n * k * 2);
  if (bt == nullptr) return PPYB200_RAISED;
  cudaError_t e = ppyb200::launch_transpose(B, reinterpret_cast<__nv_bfloat16*>(bt), k, n, stream);
  const int32_t s = finish(e, "ppyb200_matmul_bf16 (transpose)", 1);
  if (s != PPYB200_OK) return s;
  return ppyb200_matmul_bf16_kmajor(a, reinterpret_cast<const uint16_t*>(bt), bias, c, m, n, k);
}

}  // extern "C"
