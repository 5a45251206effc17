// The f32 matmul on Blackwell tensor cores: C = A @ B (+ an epilogue) for row-major f32 A and
// B, as three tf32 products (Tf32x3Operands in gemm_sm100.cuh): a split pass writes
// [A_hi | A_lo] and [B_hi^T | B_lo^T], then the tcgen05 GEMM walks A_hi.B_hi, A_hi.B_lo and
// A_lo.B_hi as one product of depth 3 Kp. The CUDA-core kernel of gemm_simt.cuh stands by for
// inputs that are not finite.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_simt.cuh"
#include "gemm_sm100.cuh"

namespace ppyb200 {
namespace gemm {

// ---- f32 operands: three tf32 products (Tf32x3Operands)

// x rounded to tf32 (10 stored significand bits, round to nearest, ties away from zero): the
// PTX conversion, whose result keeps the f32 layout with the low 13 bits zero.
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// The split of one value: hi = x rounded to tf32, lo = (x - hi) rounded to tf32 (x - hi is
// exact in f32). A value that is not finite, or rounds to one, keeps its hi alone (lo 0), so
// that an infinity or a NaN reaches the product once, as in an f32 product.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = round_tf32(x);
  lo = isfinite(hi) ? round_tf32(x - hi) : 0.f;
}

// Kp: K rounded up to a whole number of 32-wide K-steps, at least one (K = 0 splits into one
// K-step of zeros, so the product is the empty sum).
inline int64_t tf32_depth(int64_t k) { return k > 0 ? (k + 31) / 32 * 32 : 32; }

// a [m, k] row-major f32 -> a2 [m, 2 kp] = [a_hi | a_lo], zero in the columns k .. kp-1 of
// each half. Four consecutive columns per thread (kp % 4 == 0), 16-byte stores.
static __global__ void __launch_bounds__(256) split_rows_tf32_kernel(const float* __restrict__ a,
                                                             float* __restrict__ a2, int64_t m,
                                                             int64_t k, int64_t kp,
                                                             int32_t* nonfinite) {
  const int64_t quads = kp / 4;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < m * quads;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = q / quads, c = (q - row * quads) * 4;
    float hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x = c + j < k ? __ldg(a + row * k + c + j) : 0.f;
      if (!isfinite(x)) *nonfinite = 1;
      split_tf32(x, hi[j], lo[j]);
    }
    float* dst = a2 + row * 2 * kp + c;
    *reinterpret_cast<float4*>(dst) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<float4*>(dst + kp) = make_float4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// b [k, n] row-major f32 -> b2t [n, 2 kp] = [b_hi^T | b_lo^T] (K-major, zero in the columns
// k .. kp-1 of each half): 32 x 32 tiles turned through shared memory, reads coalesced along
// n and writes along k. Block 32 x 8; grid (kp / 32, ceil(n / 32)).
static __global__ void __launch_bounds__(256) split_cols_tf32_kernel(const float* __restrict__ b,
                                                             float* __restrict__ b2t, int64_t k,
                                                             int64_t n, int64_t kp,
                                                             int32_t* nonfinite) {
  __shared__ float hi_t[32][33];
  __shared__ float lo_t[32][33];
  const int64_t k0 = (int64_t)blockIdx.x * 32, n0 = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t kk = k0 + ty + 8 * j, nn = n0 + tx;
    const float x = kk < k && nn < n ? __ldg(b + kk * n + nn) : 0.f;
    if (!isfinite(x)) *nonfinite = 1;
    split_tf32(x, hi_t[ty + 8 * j][tx], lo_t[ty + 8 * j][tx]);
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t nn = n0 + ty + 8 * j, kk = k0 + tx;
    if (nn < n) {
      b2t[nn * 2 * kp + kk] = hi_t[tx][ty + 8 * j];
      b2t[nn * 2 * kp + kp + kk] = lo_t[tx][ty + 8 * j];
    }
  }
}

// Bytes of work space for an [m, k] @ [k, n] f32 product: the split operands a2 and b2t,
// then (256-byte aligned) the int32 flag the split raises on a value that is not finite.
inline int64_t tf32x3_operand_bytes(int64_t m, int64_t n, int64_t k) {
  return (m + n) * 2 * tf32_depth(k) * (int64_t)sizeof(float);
}
inline int64_t tf32x3_work_bytes(int64_t m, int64_t n, int64_t k) {
  return (tf32x3_operand_bytes(m, n, k) + 255) / 256 * 256 + 256;
}

// C = A @ B (+ the epilogue) for row-major f32 A [m, k] and B [k, n] on the tensor cores, as
// three tf32 products: split A and B into `work` (tf32x3_work_bytes(m, n, k) bytes, 256-byte
// aligned), then the GEMM with the tf32x3 operands -- CTA pairs or one CTA per tile as `launch`
// picks them. An infinity among the inputs would meet a zero low part in one of the three
// products and give NaN where the f32 loop gives an infinity, so the split raises a flag on
// any value that is not finite, and a CUDA-core kernel queued after the GEMM recomputes C
// with f32 FMAs in k order when the flag is up (it returns at once otherwise): non-finite
// inputs get IEEE f32 results. Four launches and a 4-byte memset on `stream`.
template <class Epi>
inline cudaError_t launch_tf32x3(const float* a, const float* b, float* work, int64_t m,
                                 int64_t n, int64_t k, Epi epi, int32_t* status, int sm_count,
                                 cudaStream_t stream) {
  const int64_t kp = tf32_depth(k);
  // the split's column grid and the CUDA-core recompute's row grid are 2-D launches
  if ((n + 31) / 32 > 65535 || (m + 31) / 32 > 65535) return cudaErrorInvalidValue;
  float* a2 = work;
  float* b2t = work + m * 2 * kp;
  int32_t* nonfinite = reinterpret_cast<int32_t*>(
      reinterpret_cast<char*>(work) + (tf32x3_operand_bytes(m, n, k) + 255) / 256 * 256);
  cudaError_t e = cudaMemsetAsync(nonfinite, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return e;
  int64_t blocks = (m * (kp / 4) + 255) / 256;
  if (blocks > (int64_t)sm_count * 16) blocks = (int64_t)sm_count * 16;
  if (blocks < 1) blocks = 1;
  split_rows_tf32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a, a2, m, k, kp, nonfinite);
  split_cols_tf32_kernel<<<dim3((unsigned)(kp / 32), (unsigned)((n + 31) / 32)), dim3(32, 8), 0,
                           stream>>>(b, b2t, k, n, kp, nonfinite);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int32_t form = ppyb200_gemm_form();
  if (form == PPYB200_GEMM_PAIRS || (form == PPYB200_GEMM_BY_SHAPE && m >= 2 * BM))
    e = launch_pair_op<Tf32x3Operands>(a2, b2t, m, n, kp, epi, status, stream);
  else
    e = launch_single_op<Tf32x3Operands>(a2, b2t, m, n, kp, epi, status, sm_count, stream);
  if (e != cudaSuccess) return e;
  return simt::launch(a, b, m, n, k, epi, stream, nonfinite);
}

}  // namespace gemm
}  // namespace ppyb200
