// Measurement kernels for the benchmark's rooflines (C ABI in include/ppyb200.h).
//
// ppyb200_collatz_step_peak: the issue ceiling of the Collatz step body the backend generates
// for the parallel.range reduction (tests/golden/collatz.ppyir, the reference's
// collatz_sum__par1): per step, the x != 1 test, the parity test, x / 2 or the checked 3x + 1
// (a 64-bit multiply and add, each with its overflow test), the checked step count and the
// loop-trip bound. Here every lane runs four independent chains of that step, branch-free and
// for the same number of steps, so nothing diverges, nothing waits on memory and every chain
// has work until the end -- the rate the real reduction would reach if its lanes' Collatz paths
// were all equally long. The real kernel's fraction of it is what divergence and the uneven
// path lengths cost.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ppyb200.h"
#include "ppyb200_device.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kChains = 4;

__global__ void __launch_bounds__(kThreads) collatz_step_peak_kernel(int64_t steps,
                                                                    int64_t* checksum) {
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t x[kChains], count[kChains];
  uint32_t trips = 0, bad = 0;
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    x[c] = ((id * kChains + c) << 8) | 27;  // odd starts with long paths
    count[c] = 0;
  }
  for (int64_t i = 0; i < steps; ++i) {
    if (++trips > PPYB200_LOOP_LIMIT) bad |= 16u;
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
      const int64_t v = x[c];
      bad |= (v == 1) ? 1u : 0u;
      int64_t tripled, next;
      bad |= ppyb200::mul_overflows(v, 3, &tripled) ? 2u : 0u;
      bad |= ppyb200::add_overflows(tripled, 1, &next) ? 4u : 0u;
      x[c] = (v & 1) ? next : (v >> 1);
      int64_t counted;
      bad |= ppyb200::add_overflows(count[c], 1, &counted) ? 8u : 0u;
      count[c] = counted;
    }
  }
  int64_t sum = (int64_t)trips + bad;
#pragma unroll
  for (int c = 0; c < kChains; ++c) sum += x[c] + count[c];
  // one store per block keeps every chain live without a global hot spot
  if (sum == 0x7fffffffffffffffLL) atomicAdd(reinterpret_cast<unsigned long long*>(checksum), 1ull);
}

}  // namespace

extern "C" int32_t ppyb200_collatz_step_peak(int64_t steps_per_chain, int64_t* checksum,
                                             int64_t* total_steps) {
  if (steps_per_chain < 1 || checksum == nullptr || total_steps == nullptr) {
    ppyb200_set_error("ppyb200_collatz_step_peak: steps >= 1 and device/host pointers");
    return PPYB200_RAISED;
  }
  int resident = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, collatz_step_peak_kernel,
                                                                kThreads, 0);
  if (e != cudaSuccess) return ppyb200_check((int32_t)e, "ppyb200_collatz_step_peak");
  const int64_t blocks = (int64_t)ppyb200_sm_count() * (resident > 0 ? resident : 1);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(ppyb200_stream());
  collatz_step_peak_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(steps_per_chain, checksum);
  e = cudaGetLastError();
  if (e != cudaSuccess) return ppyb200_check((int32_t)e, "ppyb200_collatz_step_peak");
  ppyb200_count_launches(1);
  *total_steps = blocks * kThreads * kChains * steps_per_chain;
  return PPYB200_OK;
}
