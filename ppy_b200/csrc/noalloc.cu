// A column reduction that allocates nothing: out[c] = max over rows r of |x[r, c]|, the
// fold `tensor.reduce(tensor.unary(x, "abs"), axes=(0,), op="max")` the b200 backend builds
// for a leading-axis reduction, with its partial results kept in a fixed device array
// instead of the runtime's scratch arena.
//
// Why: some callers cannot allocate device memory when they call -- a host application
// that reserves all of its device memory at start-up and forbids allocation afterwards
// (a latency-bound serving loop, a process sharing the GPU under a fixed budget), or code
// running under another framework's allocator that must not be bypassed. Every other
// entry point may grow the per-stream scratch arena with cudaMalloc on its first call of
// a size; this one never does.
//
// The partials live in `g_colmax_partials`, a file-scope __device__ array of
// PPYB200_NOALLOC_PARTIALS floats (1 MiB). Every GPU that loads this library holds it
// until the process exits. A call needs one partial per (row chunk, column); the number of
// chunks is chosen so that chunks x cols fits, so any row count works, and a row wider
// than PPYB200_NOALLOC_PARTIALS columns is refused before anything is launched.
//
// In host code the array's name is not a device address: it is looked up with
// cudaGetSymbolAddress while the device is current, once per device, and reused. CUDA loads
// a library's device code lazily, and the lookup is what loads this file's module -- the
// array included -- onto the device, which takes device memory. So ppyb200_init does the
// lookup (and loads both kernels) for the device it binds: after it, a call allocates
// nothing at all, not even through the driver. A caller that never runs ppyb200_init gets
// the lookup in its first call on each device instead; that call should then come before
// any stream capture and before the caller reserves its device memory.
// All calls share the one array and it keeps the previous call's contents:
// each call writes every partial it later reads, so nothing has to start at zero, but calls
// whose kernels overlap on the GPU (e.g. on two streams at once) race on it.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "../../include/ppyb200.h"
#include "ppyb200_device.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_colmax_partials[PPYB200_NOALLOC_PARTIALS];

std::mutex g_lock;
float* g_partials[kMaxDevices] = {};


// Fold |x| over the rows of one chunk for one column; every (chunk, column) partial is
// written, the identity (-inf) when the chunk holds no rows.
__global__ void __launch_bounds__(kThreads) colmax_partial(const float* __restrict__ x,
                                                           int64_t rows, int64_t cols,
                                                           int64_t rows_per_chunk,
                                                           float* __restrict__ partials) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  float acc = -INFINITY;
  for (int64_t r = r0; r < r1; ++r) acc = ppyb200::ext_max(acc, fabsf(x[r * cols + c]));
  partials[(int64_t)blockIdx.y * cols + c] = acc;
}

__global__ void __launch_bounds__(kThreads) colmax_final(const float* __restrict__ partials,
                                                         int64_t chunks, int64_t cols,
                                                         float* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float acc = -INFINITY;
  for (int64_t k = 0; k < chunks; ++k) acc = ppyb200::ext_max(acc, partials[k * cols + c]);
  out[c] = acc;
}

// The device address of g_colmax_partials on the current device `device`, looked up once
// per device; the first lookup also loads both kernels (cudaFuncGetAttributes), so that their
// first launch loads nothing either.
float* partials_address(int device) {
  std::lock_guard<std::mutex> hold(g_lock);
  if (g_partials[device] == nullptr) {
    void* address = nullptr;
    cudaError_t error = cudaGetSymbolAddress(&address, g_colmax_partials);
    if (error != cudaSuccess) {
      ppyb200_check((int32_t)error, "ppyb200_colmax_abs_f32_noalloc: cudaGetSymbolAddress");
      return nullptr;
    }
    cudaFuncAttributes attributes;
    error = cudaFuncGetAttributes(&attributes, colmax_partial);
    if (error == cudaSuccess) error = cudaFuncGetAttributes(&attributes, colmax_final);
    if (error != cudaSuccess) {
      ppyb200_check((int32_t)error, "ppyb200_colmax_abs_f32_noalloc: loading its kernels");
      return nullptr;
    }
    g_partials[device] = static_cast<float*>(address);
  }
  return g_partials[device];
}

}  // namespace

namespace ppyb200 {

// Called by ppyb200_init with `device` current: load the module of this file on the device
// and record the array's address there, so that no later call allocates.
int32_t noalloc_prepare(int device) {
  if (device < 0 || device >= kMaxDevices) {
    ppyb200_set_error("ppyb200_colmax_abs_f32_noalloc: no such device");
    return PPYB200_RAISED;
  }
  return partials_address(device) != nullptr ? PPYB200_OK : PPYB200_RAISED;
}

}  // namespace ppyb200

extern "C" int32_t ppyb200_colmax_abs_f32_noalloc(const float* x, int64_t rows, int64_t cols,
                                                  float* out) {
  if (rows < 0 || cols < 0) {
    ppyb200_set_error("ppyb200_colmax_abs_f32_noalloc: negative extent");
    return PPYB200_RAISED;
  }
  if (cols > PPYB200_NOALLOC_PARTIALS) {
    ppyb200_set_error(
        "ppyb200_colmax_abs_f32_noalloc: a row of more than PPYB200_NOALLOC_PARTIALS (262144) "
        "columns does not fit the static scratch array; use the allocating entry point");
    return PPYB200_RAISED;
  }
  if (cols == 0) return PPYB200_OK;
  int device = 0;
  const cudaError_t got = cudaGetDevice(&device);
  if (got != cudaSuccess) return ppyb200_check((int32_t)got, "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) {
    ppyb200_set_error("ppyb200_colmax_abs_f32_noalloc: no such device");
    return PPYB200_RAISED;
  }
  float* partials = partials_address(device);
  if (partials == nullptr) return PPYB200_RAISED;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  const int64_t col_blocks = (cols + kThreads - 1) / kThreads;
  // enough row chunks to fill the SMs, no more than the array holds for this width
  int64_t chunks = ((int64_t)ppyb200_sm_count() * 8 + col_blocks - 1) / col_blocks;
  const int64_t fit = PPYB200_NOALLOC_PARTIALS / cols;
  if (chunks > fit) chunks = fit;
  if (chunks > rows) chunks = rows;
  if (chunks > 65535) chunks = 65535;
  if (chunks < 1) chunks = 1;
  const int64_t rows_per_chunk = rows > 0 ? (rows + chunks - 1) / chunks : 1;
  chunks = rows > 0 ? (rows + rows_per_chunk - 1) / rows_per_chunk : 1;
  colmax_partial<<<dim3((unsigned)col_blocks, (unsigned)chunks), kThreads, 0, stream>>>(
      x, rows, cols, rows_per_chunk, partials);
  colmax_final<<<(unsigned)col_blocks, kThreads, 0, stream>>>(partials, chunks, cols, out);
  const cudaError_t launched = cudaGetLastError();
  if (launched != cudaSuccess)
    return ppyb200_check((int32_t)launched, "ppyb200_colmax_abs_f32_noalloc: launch");
  ppyb200_count_launches(2);
  return PPYB200_OK;
}
