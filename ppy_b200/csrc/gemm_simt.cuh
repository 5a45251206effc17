// A plain tiled matmul on the CUDA cores for the shapes and element types the tensor-core
// kernel does not take (f32 operands, or bf16 shapes that are not whole 128x256x64 tiles):
// D[M,N] = A[M,K] @ B[K,N] with row-major A and B, f32 accumulation with FMAs in k order,
// then the same elementwise epilogue as the tensor-core kernel.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ppyb200_device.cuh"

namespace ppyb200 {
namespace simt {

constexpr int TILE = 32;

template <class T>
__device__ __forceinline__ float to_f32(T v) {
  return ppyb200::convert<float, T>(v);
}

// A 32x32 output tile per 32x8 block; every thread computes 4 outputs of one column. With
// `only_if` given, the kernel does nothing unless *only_if is nonzero (a recomputation that
// an earlier kernel on the stream asks for).
template <class T, class Epi>
__global__ void __launch_bounds__(256) matmul_kernel(const T* __restrict__ a,
                                                     const T* __restrict__ b, int64_t m,
                                                     int64_t n, int64_t k, Epi epi,
                                                     const int32_t* only_if) {
  if (only_if != nullptr && *(volatile const int32_t*)only_if == 0) return;
  __shared__ float as[TILE][TILE + 1];
  __shared__ float bs[TILE][TILE + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const int64_t row0 = (int64_t)blockIdx.y * TILE, col0 = (int64_t)blockIdx.x * TILE;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t k0 = 0; k0 < k; k0 += TILE) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty + 8 * i;
      const int64_t ar = row0 + r, ac = k0 + tx;
      as[r][tx] = (ar < m && ac < k) ? to_f32(a[ar * k + ac]) : 0.f;
      const int64_t br = k0 + r, bc = col0 + tx;
      bs[r][tx] = (br < k && bc < n) ? to_f32(b[br * n + bc]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int q = 0; q < TILE; ++q) {
      const float bv = bs[q][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(as[ty + 8 * i][q], bv, acc[i]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + ty + 8 * i, col = col0 + tx;
    if (row < m && col < n) epi.store(acc[i], row, col);
  }
}

template <class T, class Epi>
inline cudaError_t launch(const T* a, const T* b, int64_t m, int64_t n, int64_t k, Epi epi,
                          cudaStream_t stream, const int32_t* only_if = nullptr) {
  if (m <= 0 || n <= 0) return cudaSuccess;
  dim3 grid((unsigned)((n + TILE - 1) / TILE), (unsigned)((m + TILE - 1) / TILE));
  matmul_kernel<T, Epi><<<grid, dim3(32, 8), 0, stream>>>(a, b, m, n, k, epi, only_if);
  return cudaGetLastError();
}

}  // namespace simt

// [rows, cols] -> [cols, rows] through 32x32 shared-memory tiles (coalesced both ways).
template <class T>
__global__ void __launch_bounds__(256) transpose_kernel(const T* __restrict__ in,
                                                        T* __restrict__ out, int64_t rows,
                                                        int64_t cols) {
  __shared__ T tile[32][33];
  const int64_t c0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + threadIdx.y + 8 * i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[threadIdx.y + 8 * i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = c0 + threadIdx.y + 8 * i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][threadIdx.y + 8 * i];
  }
}

template <class T>
inline cudaError_t launch_transpose(const T* in, T* out, int64_t rows, int64_t cols,
                                    cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  transpose_kernel<T><<<grid, dim3(32, 8), 0, stream>>>(in, out, rows, cols);
  return cudaGetLastError();
}

}  // namespace ppyb200
