// The tensor-parallel exchange of GPT-2's row-parallel layers over NVLink, fused into the
// GEMM: the reduction that the NCCL path does with an all-reduce after the GEMM
// (x <- x + bias + sum over ranks of a_r @ w_r^T).
//
//   ppyb200_tp_partial_scatter   this rank's partial product a_r @ w_r^T on tcgen05 tensor
//                                cores; the epilogue stores every 16-byte piece of it into
//                                slot r of every rank's exchange buffer (peer memory, mapped
//                                through CUDA IPC), so the transfer overlaps the tiles still
//                                being multiplied
//   ppyb200_tp_signal            after it on the stream: epoch into flag r of every rank
//   ppyb200_tp_accumulate        waits (bounded) for every rank's flag to reach the epoch,
//                                then x += bias + slot 0 + slot 1 + ... in rank order, so
//                                every rank sums the same values in the same order and the
//                                residual stream stays bit-identical across the group
//
// The host double-buffers the slots by the parity of the epoch: a rank writes parity p for
// epoch E only after its own wait for E - 1, which needs every peer's flag for E - 1, which a
// peer raises after its accumulate of E - 2 -- the last read of parity p. No load anywhere is
// a TMA multicast: the peer traffic is plain stores from the epilogue and the flag stores.
//
// The reduce-scatter form sends each rank (R - 1) / R of the partial twice instead of all of
// it R - 1 times: rows split into R blocks, block s owned by rank s.
//
//   ppyb200_tp_partial_reduce_scatter   the GEMM's epilogue stores the tile rows of block s
//                                       into slot r of rank s's exchange buffer only
//   ppyb200_tp_signal                   flags of the first round
//   ppyb200_tp_reduce_block             waits for them; x[own block] += bias + slot 0 + slot 1
//                                       + ... in rank order, and the summed block goes into
//                                       slot r of every rank's gather buffer
//   ppyb200_tp_signal                   flags of the second round
//   ppyb200_tp_gather_blocks            waits for them; the other ranks' blocks into x
// Each block is summed once, by its owner, in the same order as the all-slot form: the
// residual stream stays bit-identical across the group and equal to that form's. Both buffers
// are double-buffered by epoch parity as above: a rank writes parity p of epoch E after its
// gather wait of E - 1, which follows every peer's reduce of E - 1 and so its reads of E - 2.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "../../include/ppyb200.h"
#include "gemm_sm100.cuh"
#include "ppyb200_device.cuh"

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaStream_t stream_now() { return reinterpret_cast<cudaStream_t>(ppyb200_stream()); }

int32_t finish(cudaError_t error, const char* what, uint64_t launched) {
  if (error != cudaSuccess) return ppyb200_check((int32_t)error, what);
  ppyb200_count_launches(launched);
  return PPYB200_OK;
}

constexpr int MAX_RANKS = 8;
// A wait gives up after this many nanoseconds (globaltimer): a peer that stopped or never came
constexpr uint64_t WAIT_NS = 2000000000ull;

// The partial product's four-column quads, written to slot `rank` of every rank's buffer:
// dst[s] is that slot in rank s's buffer (this device's own, or a peer's mapped here).
struct PeerScatterQuads {
  static constexpr bool kQuads = true;
  float* dst[MAX_RANKS];
  int32_t ranks;
  int64_t ld;
  __device__ __forceinline__ void store_quads(const float4 (&v)[8], int64_t row, int count,
                                              int64_t col) const {
#pragma unroll
    for (int s = 0; s < MAX_RANKS; ++s) {
      if (s >= ranks) break;
      float* p = dst[s] + row * ld + col;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < count) *reinterpret_cast<float4*>(p + 4 * i * ld) = v[i];
    }
  }
};

// The partial product's quads, each row to the rank that owns its block (rows
// [s * block_rows, (s + 1) * block_rows) to rank s): dst[s] is this rank's slot in rank s's
// exchange buffer, [block_rows, ld] f32.
struct PeerScatterBlocks {
  static constexpr bool kQuads = true;
  float* dst[MAX_RANKS];
  int64_t block_rows;
  int64_t ld;
  __device__ __forceinline__ void store_quads(const float4 (&v)[8], int64_t row, int count,
                                              int64_t col) const {
    int64_t s = row / block_rows, start = s * block_rows;  // one division for the 8 rows
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i >= count) break;
      const int64_t r = row + 4 * i;
      while (r >= start + block_rows) {  // at most ranks - 1 steps over the 29 rows
        ++s;
        start += block_rows;
      }
      *reinterpret_cast<float4*>(dst[s] + (r - start) * ld + col) = v[i];
    }
  }
};

struct FlagSet {
  int32_t* flag[MAX_RANKS];
};

__global__ void tp_signal_kernel(FlagSet flags, int32_t ranks, int32_t rank, int32_t epoch) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  // the GEMM before this kernel on the stream wrote the slots; publish them system-wide, then
  // the flags (release stores: a peer that reads the epoch also sees the slots)
  asm volatile("fence.sc.sys;" ::: "memory");
  for (int s = 0; s < ranks; ++s)
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(flags.flag[s] + rank), "r"(epoch)
                 : "memory");
}

__device__ __forceinline__ int32_t load_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A 16-byte load of memory that peers store into while this kernel runs: relaxed at system
// scope, never through the non-coherent (read-only) cache path that a const __restrict__
// pointer would let the compiler choose. Ordered after the peers' stores by the waiting
// thread's ld.acquire.sys of their flags and the __syncthreads that follows it.
__device__ __forceinline__ float4 load_peer4(const float* p) {
  float4 v;
  asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// x[M,N] += bias[N] + sum_r exchange[r][M,N], after every flag reaches `epoch`. float4 per
// thread (N % 4 == 0), grid-stride; one thread per block waits, the block follows it.
// `exchange` is written by the peers up to the flags this kernel waits on, so it is read
// with load_peer4, never as read-only data.
__global__ void __launch_bounds__(256) tp_accumulate_kernel(
    float* __restrict__ x, const float* __restrict__ bias, const float* exchange,
    const int32_t* flags, int32_t ranks, int64_t m, int64_t n, int32_t epoch,
    int32_t* status) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    const uint64_t start = global_ns();
    int ok = 1;
    for (int s = 0; s < ranks && ok; ++s) {
      while (load_acquire_sys(flags + s) < epoch) {
        if (global_ns() - start > WAIT_NS) {
          ok = 0;
          break;
        }
        __nanosleep(200);
      }
    }
    if (!ok && status != nullptr) atomicMax(status, PPYB200_DEVICE_RAISED);
    ready = ok;
  }
  __syncthreads();
  if (!ready) return;
  const int64_t quads = m * n / 4, per = n / 4, slot = m * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = *reinterpret_cast<const float4*>(x + 4 * i);
    const float4 b = bias != nullptr ? __ldg(reinterpret_cast<const float4*>(bias) + i % per)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 sum = b;
    for (int s = 0; s < ranks; ++s) {
      const float4 p = load_peer4(exchange + s * slot + 4 * i);
      sum.x += p.x;
      sum.y += p.y;
      sum.z += p.z;
      sum.w += p.w;
    }
    acc.x += sum.x;
    acc.y += sum.y;
    acc.z += sum.z;
    acc.w += sum.w;
    *reinterpret_cast<float4*>(x + 4 * i) = acc;
  }
}

// Bounded wait of one thread for flags[0..ranks) to reach `epoch`; the block follows it.
__device__ __forceinline__ bool block_wait_flags(const int32_t* flags, int32_t ranks,
                                                 int32_t epoch, int32_t* status) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    const uint64_t start = global_ns();
    int ok = 1;
    for (int s = 0; s < ranks && ok; ++s) {
      while (load_acquire_sys(flags + s) < epoch) {
        if (global_ns() - start > WAIT_NS) {
          ok = 0;
          break;
        }
        __nanosleep(200);
      }
    }
    if (!ok && status != nullptr) atomicMax(status, PPYB200_DEVICE_RAISED);
    ready = ok;
  }
  __syncthreads();
  return ready != 0;
}

struct PeerBlocks {
  float* dst[MAX_RANKS];
};

// x[rows of block `rank`] += bias + sum_s exchange[s] (rank order), after every flag reaches
// `epoch`; the result also into gather[s] (this rank's slot in rank s's gather buffer) for
// every s != rank. exchange: this rank's [ranks][block_rows, n] slots (peers store into it).
__global__ void __launch_bounds__(256) tp_reduce_block_kernel(
    float* __restrict__ x, const float* __restrict__ bias, const float* exchange, PeerBlocks gather,
    const int32_t* flags, int32_t ranks, int32_t rank, int64_t m, int64_t n, int64_t block_rows,
    int32_t epoch, int32_t* status) {
  if (!block_wait_flags(flags, ranks, epoch, status)) return;
  const int64_t first = rank * block_rows;
  const int64_t rows = (m - first < block_rows ? m - first : block_rows);
  if (rows <= 0) return;
  const int64_t quads = rows * n / 4, per = n / 4, slot = block_rows * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = *reinterpret_cast<const float4*>(x + first * n + 4 * i);
    const float4 b = bias != nullptr ? __ldg(reinterpret_cast<const float4*>(bias) + i % per)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 sum = b;
    for (int s = 0; s < ranks; ++s) {
      const float4 p = load_peer4(exchange + s * slot + 4 * i);
      sum.x += p.x;
      sum.y += p.y;
      sum.z += p.z;
      sum.w += p.w;
    }
    acc.x += sum.x;
    acc.y += sum.y;
    acc.z += sum.z;
    acc.w += sum.w;
    *reinterpret_cast<float4*>(x + first * n + 4 * i) = acc;
    for (int s = 0; s < ranks; ++s)
      if (s != rank) *reinterpret_cast<float4*>(gather.dst[s] + 4 * i) = acc;
  }
}

// After every flag reaches `epoch`: the blocks of the other ranks from this rank's gather
// buffer ([ranks][block_rows, n], slot s written by rank s) into x.
__global__ void __launch_bounds__(256) tp_gather_blocks_kernel(
    float* __restrict__ x, const float* gathered, const int32_t* flags, int32_t ranks,
    int32_t rank, int64_t m, int64_t n, int64_t block_rows, int32_t epoch, int32_t* status) {
  if (!block_wait_flags(flags, ranks, epoch, status)) return;
  const int64_t per_block = block_rows * n / 4;
  const int64_t quads = (int64_t)ranks * per_block;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / per_block, q = i - s * per_block;
    if (s == rank) continue;
    const int64_t row = s * block_rows + (4 * q) / n;
    if (row >= m) continue;
    *reinterpret_cast<float4*>(x + s * block_rows * n + 4 * q) =
        load_peer4(gathered + s * block_rows * n + 4 * q);
  }
}

}  // namespace

extern "C" {

void* ppyb200_shared_alloc(int64_t bytes, uint8_t* handle) {
  if (bytes <= 0 || handle == nullptr) {
    ppyb200_set_error("ppyb200_shared_alloc: a positive size and a handle buffer");
    return nullptr;
  }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) {
    ppyb200_check((int32_t)e, "ppyb200_shared_alloc");
    return nullptr;
  }
  e = cudaMemset(p, 0, (size_t)bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    ppyb200_check((int32_t)e, "ppyb200_shared_alloc: IPC handle");
    return nullptr;
  }
  memcpy(handle, &h, sizeof(h));
  return p;
}

void ppyb200_shared_free(void* pointer) {
  if (pointer != nullptr) cudaFree(pointer);
}

void* ppyb200_shared_open(const uint8_t* handle) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    ppyb200_check((int32_t)e, "ppyb200_shared_open");
    return nullptr;
  }
  return p;
}

void ppyb200_shared_close(void* pointer) {
  if (pointer != nullptr) cudaIpcCloseMemHandle(pointer);
}

int32_t ppyb200_tp_partial_scatter(const uint16_t* a, const uint16_t* w, float* const* slots,
                                   int32_t ranks, int64_t m, int64_t n, int64_t k,
                                   int32_t* status) {
  if (m < 0 || n < 0 || k < 0 || ranks < 1 || ranks > MAX_RANKS || slots == nullptr) {
    ppyb200_set_error("ppyb200_tp_partial_scatter: extents >= 0 and 1 to 8 ranks");
    return PPYB200_RAISED;
  }
  if (m == 0 || n == 0) return PPYB200_OK;
  if (!ppyb200::gemm::tileable(m, n, k) || n % 4 != 0 || !aligned16(a) || !aligned16(w)) {
    ppyb200_set_error("ppyb200_tp_partial_scatter: K % 64, N % 4 and 16-byte aligned operands");
    return PPYB200_RAISED;
  }
  PeerScatterQuads epi{};
  for (int s = 0; s < ranks; ++s) {
    if (slots[s] == nullptr || !aligned16(slots[s])) {
      ppyb200_set_error("ppyb200_tp_partial_scatter: 16-byte aligned slots");
      return PPYB200_RAISED;
    }
    epi.dst[s] = slots[s];
  }
  epi.ranks = ranks;
  epi.ld = n;
  cudaError_t e = ppyb200::gemm::launch(reinterpret_cast<const __nv_bfloat16*>(a),
                                        reinterpret_cast<const __nv_bfloat16*>(w), m, n, k, epi,
                                        status, ppyb200_sm_count(), stream_now());
  return finish(e, "ppyb200_tp_partial_scatter", 1);
}

int32_t ppyb200_tp_signal(int32_t* const* flags, int32_t ranks, int32_t rank, int32_t epoch) {
  if (ranks < 1 || ranks > MAX_RANKS || rank < 0 || rank >= ranks || flags == nullptr) {
    ppyb200_set_error("ppyb200_tp_signal: 1 to 8 ranks and a rank among them");
    return PPYB200_RAISED;
  }
  FlagSet set{};
  for (int s = 0; s < ranks; ++s) set.flag[s] = flags[s];
  tp_signal_kernel<<<1, 32, 0, stream_now()>>>(set, ranks, rank, epoch);
  return finish(cudaGetLastError(), "ppyb200_tp_signal", 1);
}

int32_t ppyb200_tp_accumulate(float* x, const float* bias, const float* exchange,
                              const int32_t* flags, int32_t ranks, int64_t m, int64_t n,
                              int32_t epoch, int32_t* status) {
  if (ranks < 1 || ranks > MAX_RANKS || m < 0 || n <= 0 || n % 4 != 0 || !aligned16(x) ||
      !aligned16(exchange) || (bias != nullptr && !aligned16(bias)) || flags == nullptr) {
    ppyb200_set_error("ppyb200_tp_accumulate: N % 4 == 0, 16-byte aligned x, bias, exchange");
    return PPYB200_RAISED;
  }
  if (m == 0) return PPYB200_OK;
  const int64_t quads = m * n / 4;
  int64_t blocks = (quads + 255) / 256;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  tp_accumulate_kernel<<<(unsigned)blocks, 256, 0, stream_now()>>>(x, bias, exchange, flags,
                                                                   ranks, m, n, epoch, status);
  return finish(cudaGetLastError(), "ppyb200_tp_accumulate", 1);
}

int32_t ppyb200_tp_partial_reduce_scatter(const uint16_t* a, const uint16_t* w,
                                          float* const* slots, int32_t ranks, int64_t m,
                                          int64_t n, int64_t k, int32_t* status) {
  if (m < 0 || n < 0 || k < 0 || ranks < 1 || ranks > MAX_RANKS || slots == nullptr) {
    ppyb200_set_error("ppyb200_tp_partial_reduce_scatter: extents >= 0 and 1 to 8 ranks");
    return PPYB200_RAISED;
  }
  if (m == 0 || n == 0) return PPYB200_OK;
  if (!ppyb200::gemm::tileable(m, n, k) || n % 4 != 0 || !aligned16(a) || !aligned16(w)) {
    ppyb200_set_error(
        "ppyb200_tp_partial_reduce_scatter: K % 64, N % 4 and 16-byte aligned operands");
    return PPYB200_RAISED;
  }
  PeerScatterBlocks epi{};
  for (int s = 0; s < ranks; ++s) {
    if (slots[s] == nullptr || !aligned16(slots[s])) {
      ppyb200_set_error("ppyb200_tp_partial_reduce_scatter: 16-byte aligned slots");
      return PPYB200_RAISED;
    }
    epi.dst[s] = slots[s];
  }
  epi.block_rows = (m + ranks - 1) / ranks;
  epi.ld = n;
  cudaError_t e = ppyb200::gemm::launch(reinterpret_cast<const __nv_bfloat16*>(a),
                                        reinterpret_cast<const __nv_bfloat16*>(w), m, n, k, epi,
                                        status, ppyb200_sm_count(), stream_now());
  return finish(e, "ppyb200_tp_partial_reduce_scatter", 1);
}

int32_t ppyb200_tp_reduce_block(float* x, const float* bias, const float* exchange,
                                float* const* gather, const int32_t* flags, int32_t ranks,
                                int32_t rank, int64_t m, int64_t n, int32_t epoch,
                                int32_t* status) {
  if (ranks < 1 || ranks > MAX_RANKS || rank < 0 || rank >= ranks || m < 0 || n <= 0 ||
      n % 4 != 0 || !aligned16(x) || !aligned16(exchange) ||
      (bias != nullptr && !aligned16(bias)) || flags == nullptr || gather == nullptr) {
    ppyb200_set_error("ppyb200_tp_reduce_block: 1 to 8 ranks, N % 4 == 0, 16-byte aligned x, "
                      "bias, exchange");
    return PPYB200_RAISED;
  }
  if (m == 0) return PPYB200_OK;
  PeerBlocks peers{};
  for (int s = 0; s < ranks; ++s) {
    if (s != rank && (gather[s] == nullptr || !aligned16(gather[s]))) {
      ppyb200_set_error("ppyb200_tp_reduce_block: 16-byte aligned gather slots");
      return PPYB200_RAISED;
    }
    peers.dst[s] = gather[s];
  }
  const int64_t block_rows = (m + ranks - 1) / ranks;
  const int64_t quads = block_rows * n / 4;
  int64_t blocks = (quads + 255) / 256;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  tp_reduce_block_kernel<<<(unsigned)blocks, 256, 0, stream_now()>>>(
      x, bias, exchange, peers, flags, ranks, rank, m, n, block_rows, epoch, status);
  return finish(cudaGetLastError(), "ppyb200_tp_reduce_block", 1);
}

int32_t ppyb200_tp_gather_blocks(float* x, const float* gathered, const int32_t* flags,
                                 int32_t ranks, int32_t rank, int64_t m, int64_t n,
                                 int32_t epoch, int32_t* status) {
  if (ranks < 1 || ranks > MAX_RANKS || rank < 0 || rank >= ranks || m < 0 || n <= 0 ||
      n % 4 != 0 || !aligned16(x) || !aligned16(gathered) || flags == nullptr) {
    ppyb200_set_error("ppyb200_tp_gather_blocks: 1 to 8 ranks, N % 4 == 0, 16-byte aligned "
                      "x and gather buffer");
    return PPYB200_RAISED;
  }
  if (m == 0) return PPYB200_OK;
  const int64_t block_rows = (m + ranks - 1) / ranks;
  const int64_t quads = (int64_t)ranks * block_rows * n / 4;
  int64_t blocks = (quads + 255) / 256;
  const int64_t cap = (int64_t)ppyb200_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  tp_gather_blocks_kernel<<<(unsigned)blocks, 256, 0, stream_now()>>>(
      x, gathered, flags, ranks, rank, m, n, block_rows, epoch, status);
  return finish(cudaGetLastError(), "ppyb200_tp_gather_blocks", 1);
}

}  // extern "C"
