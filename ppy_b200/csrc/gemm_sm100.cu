// The C-ABI matmul entry points of libppyb200 (include/ppyb200.h): bf16 x bf16 -> f32 with
// an optional f32 bias row, on tcgen05 tensor cores for whole 128x256x64 tiles and on the
// CUDA cores otherwise; f32 x f32 -> f32 as three tf32 products on the tensor cores.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/ppyb200.h"
#include "gemm_sm100.cuh"
#include "gemm_f32.cuh"
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

int32_t ppyb200_matmul_bf16_kmajor_ld(const uint16_t* a, const uint16_t* bt, const float* bias,
                                      float* c, int64_t ldc, int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0 || ldc < n) {
    ppyb200_set_error("ppyb200_matmul_bf16_kmajor_ld: extents >= 0 and ldc >= N");
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
  // Deep K (the MMAs set the pace): C = A.B + bias by columns of 32 rows, each store 32
  // consecutive floats of one row (0.806 against 0.826 ms for quads at 8192^3). Shallow K
  // (the stores set it): four-column quads, a quarter of the store instructions (GPT-2's LM
  // head, 32768 x 50257 x 768 into rows 50272 apart, on CTA pairs: 2.48 ms against 2.99 for
  // columns; on one CTA per tile 2.79 against 2.92). Either form stores whole 128-byte lines
  // when rows start on one (C aligned so, ldc % 32 == 0) and splits every store over two
  // lines otherwise (3.08 ms with ldc = 50257). `launch` picks CTA pairs or one CTA per tile.
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(a);
  const auto* B = reinterpret_cast<const __nv_bfloat16*>(bt);
  cudaError_t e;
  if (k < ppyb200::gemm::DEEP_K && ldc % 4 == 0 && aligned16(c) &&
      (bias == nullptr || aligned16(bias)))
    e = ppyb200::gemm::launch(A, B, m, n, k, ppyb200::gemm::BiasQuads{bias, c, ldc, n}, status,
                              ppyb200_sm_count(), stream);
  else
    e = ppyb200::gemm::launch(A, B, m, n, k, ppyb200::gemm::BiasEpilogue{bias, c, ldc}, status,
                              ppyb200_sm_count(), stream);
  return finish(e, "ppyb200_matmul_bf16_kmajor", 1);
}

int32_t ppyb200_matmul_bf16_kmajor(const uint16_t* a, const uint16_t* bt, const float* bias,
                                   float* c, int64_t m, int64_t n, int64_t k) {
  return ppyb200_matmul_bf16_kmajor_ld(a, bt, bias, c, n, m, n, k);
}

int32_t ppyb200_matmul_f32(const float* a, const float* b, const float* bias, float* c,
                           int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) {
    ppyb200_set_error("ppyb200_matmul_f32: negative extent");
    return PPYB200_RAISED;
  }
  if (m == 0 || n == 0) return PPYB200_OK;
  const int64_t kp = ppyb200::gemm::tf32_depth(k);
  if (m >= (1ll << 31) || n >= (1ll << 31) || 2 * kp >= (1ll << 31)) {
    ppyb200_set_error("ppyb200_matmul_f32: an extent beyond the tensor maps' int32 range");
    return PPYB200_RAISED;
  }
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  int32_t* status = ppyb200_status_word();
  if (status == nullptr) return PPYB200_RAISED;
  float* work = static_cast<float*>(ppyb200_scratch(ppyb200::gemm::tf32x3_work_bytes(m, n, k)));
  if (work == nullptr) return PPYB200_RAISED;
  // (K = 0 splits into one K-step of zeros: C = bias, the empty sum, as the reference's
  // loop nest gives)
  cudaError_t e = ppyb200::gemm::launch_tf32x3(a, b, work, m, n, k,
                                               ppyb200::gemm::BiasEpilogue{bias, c, n}, status,
                                               ppyb200_sm_count(), stream);
  return finish(e, "ppyb200_matmul_f32", 4);
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
