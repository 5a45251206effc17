// Device-side building blocks shared by every kernel the b200 backend generates.
//
// Scalar semantics follow PPy's canonical IR, which is what the reference's LLVM
// backend computes on the CPU:
//   * min / max are NaN-propagating: `a` wins when it is NaN or the extreme, a NaN `c`
//     wins the comparison it fails (ir/dialects/tensor.py:691-701);
//   * integer add/sub/mul carrying overflow="python" take the fallback on int64
//     overflow (backend/llvm/from_ir.py:731-771); "wrap"/"native" wrap; "proven" wraps;
//   * integer div/mod round toward -inf by default (from_ir.py:788-833);
//   * float compares are IEEE: every compare with a NaN is false except `!=`
//     (from_ir.py:855-868).
// Reductions combine with the same operations (lower_tensor.py:1841-1870); the order of
// combination is a tree here instead of the reference's row-major fold, which changes
// floating-point rounding only (integers are exact either way).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include <atomic>
#include <mutex>
#include <utility>

extern "C" int32_t ppyb200_pdl(void);  // libppyb200: whether launches carry the PDL attribute

#define PPY_STATUS_OK 0
#define PPY_STATUS_FALLBACK 1
#define PPY_STATUS_RAISED (-1)

// Status words kernels raise (atomicMax: the most severe wins). A body that failed with
// PPY_STATUS_RAISED -- e.g. a loop past PPYB200_LOOP_LIMIT trips -- records
// PPYB200_DEVICE_RAISED; the host maps it to PPY_STATUS_RAISED with a message.
#define PPYB200_DEVICE_FALLBACK 1
#define PPYB200_DEVICE_RAISED 2
#ifndef PPYB200_LOOP_LIMIT
#define PPYB200_LOOP_LIMIT (1u << 26)
#endif

namespace ppyb200 {

// ---------------------------------------------------------------- min / max

template <class T>
__device__ __forceinline__ T ext_max(T a, T c) {
  T chosen = (a >= c) ? a : c;
  return (a == a) ? chosen : a;
}
template <class T>
__device__ __forceinline__ T ext_min(T a, T c) {
  T chosen = (a <= c) ? a : c;
  return (a == a) ? chosen : a;
}
__device__ __forceinline__ int64_t ext_max(int64_t a, int64_t c) { return a >= c ? a : c; }
__device__ __forceinline__ int64_t ext_min(int64_t a, int64_t c) { return a <= c ? a : c; }
__device__ __forceinline__ int32_t ext_max(int32_t a, int32_t c) { return a >= c ? a : c; }
__device__ __forceinline__ int32_t ext_min(int32_t a, int32_t c) { return a <= c ? a : c; }

// ---------------------------------------------------------------- checked int64

// Two's-complement add/sub/mul that report int64 overflow instead of wrapping:
// the reference's `llvm.s{add,sub,mul}.with.overflow.i64` (from_ir.py:757-771).
__host__ __device__ __forceinline__ bool add_overflows(int64_t a, int64_t b, int64_t* r) {
  int64_t s = (int64_t)((uint64_t)a + (uint64_t)b);
  *r = s;
  return ((a ^ s) & (b ^ s)) < 0;
}
__host__ __device__ __forceinline__ bool sub_overflows(int64_t a, int64_t b, int64_t* r) {
  int64_t s = (int64_t)((uint64_t)a - (uint64_t)b);
  *r = s;
  return ((a ^ b) & (a ^ s)) < 0;
}
__host__ __device__ __forceinline__ bool mul_overflows(int64_t a, int64_t b, int64_t* r) {
  int64_t lo = (int64_t)((uint64_t)a * (uint64_t)b);
#ifdef __CUDA_ARCH__
  int64_t hi = __mul64hi(a, b);
#else
  int64_t hi = (int64_t)(((__int128)a * (__int128)b) >> 64);
#endif
  *r = lo;
  return hi != (lo >> 63);
}

// Floor division and modulo (Python's `//` and `%` on ints), for a nonzero divisor.
__host__ __device__ __forceinline__ int64_t floordiv(int64_t a, int64_t b) {
  int64_t q = a / b;
  int64_t r = a % b;
  return (r != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}
__host__ __device__ __forceinline__ int64_t floormod(int64_t a, int64_t b) {
  int64_t r = a % b;
  return (r != 0 && ((a < 0) != (b < 0))) ? r + b : r;
}

// ---------------------------------------------------------------- combine ops

struct OpAdd {
  template <class T> __device__ __forceinline__ static T apply(T a, T b) { return a + b; }
};
struct OpMul {
  template <class T> __device__ __forceinline__ static T apply(T a, T b) { return a * b; }
};
struct OpMax {
  template <class T> __device__ __forceinline__ static T apply(T a, T b) { return ext_max(a, b); }
};
struct OpMin {
  template <class T> __device__ __forceinline__ static T apply(T a, T b) { return ext_min(a, b); }
};

template <class T>
__device__ __forceinline__ T shfl_xor(T v, int mask, int width) {
  return __shfl_xor_sync(0xffffffffu, v, mask, width);
}

// Butterfly over `width` lanes (a power of two <= 32): every lane ends with the value.
template <class Op, int WIDTH, class T>
__device__ __forceinline__ T group_reduce(T v) {
#pragma unroll
  for (int mask = WIDTH / 2; mask > 0; mask >>= 1) v = Op::apply(v, shfl_xor(v, mask, WIDTH));
  return v;
}

// ---------------------------------------------------------------- vector memory

// Streaming 128-bit loads and stores: each byte of a fused group's inputs is read once,
// so the loads bypass L1 allocation and the stores are marked evict-first.
__device__ __forceinline__ float4 ld_stream4(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void st_stream4(float* p, float4 v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}
__device__ __forceinline__ double2 ld_stream2(const double* p) {
  return __ldcs(reinterpret_cast<const double2*>(p));
}
__device__ __forceinline__ void st_stream2(double* p, double2 v) {
  __stcs(reinterpret_cast<double2*>(p), v);
}

// ---------------------------------------------------------------- element conversions

__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f32_to_bf16(float v) { return __float2bfloat16_rn(v); }

// `special.*` functions without a CUDA namesake.
__device__ __forceinline__ float ndtr(float x) { return normcdff(x); }
__device__ __forceinline__ double ndtr(double x) { return normcdf(x); }
__device__ __forceinline__ float logit(float x) { return logf(x / (1.0f - x)); }
__device__ __forceinline__ double logit(double x) { return log(x / (1.0 - x)); }

// Record a fallback in the call's status word; the host wrapper reads it after the launch.
__device__ __forceinline__ void raise_fallback(int32_t* status) {
  if (status != nullptr) atomicMax(status, PPYB200_DEVICE_FALLBACK);
}
// Record the status a device function returned (fallback or raised).
__device__ __forceinline__ void raise_status(int32_t* status, int32_t returned) {
  if (status != nullptr)
    atomicMax(status, returned == PPY_STATUS_FALLBACK ? PPYB200_DEVICE_FALLBACK
                                                      : PPYB200_DEVICE_RAISED);
}

}  // namespace ppyb200

namespace ppyb200 {

// ---------------------------------------------------------------- conversions

template <class To, class From>
__device__ __forceinline__ To convert(From v) { return static_cast<To>(v); }
template <> __device__ __forceinline__ float convert<float, __nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ double convert<double, __nv_bfloat16>(__nv_bfloat16 v) {
  return (double)__bfloat162float(v);
}
template <> __device__ __forceinline__ __nv_bfloat16 convert<__nv_bfloat16, float>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __nv_bfloat16 convert<__nv_bfloat16, double>(double v) {
  return __double2bfloat16(v);
}
template <> __device__ __forceinline__ __nv_bfloat16 convert<__nv_bfloat16, __nv_bfloat16>(
    __nv_bfloat16 v) {
  return v;
}
template <> __device__ __forceinline__ int64_t convert<int64_t, __nv_bfloat16>(__nv_bfloat16 v) {
  return (int64_t)__bfloat162float(v);
}

// ---------------------------------------------------------------- wrapping integer combine

// Integer reductions combine with wrapping arithmetic (lower_tensor.py:1855-1868 and
// lower_parallel.py's chunk fold use overflow="wrap"); floats combine natively.
__device__ __forceinline__ float comb_add(float a, float b) { return a + b; }
__device__ __forceinline__ double comb_add(double a, double b) { return a + b; }
__device__ __forceinline__ int64_t comb_add(int64_t a, int64_t b) {
  return (int64_t)((uint64_t)a + (uint64_t)b);
}
__device__ __forceinline__ int32_t comb_add(int32_t a, int32_t b) {
  return (int32_t)((uint32_t)a + (uint32_t)b);
}
__device__ __forceinline__ float comb_mul(float a, float b) { return a * b; }
__device__ __forceinline__ double comb_mul(double a, double b) { return a * b; }
__device__ __forceinline__ int64_t comb_mul(int64_t a, int64_t b) {
  return (int64_t)((uint64_t)a * (uint64_t)b);
}
__device__ __forceinline__ int32_t comb_mul(int32_t a, int32_t b) {
  return (int32_t)((uint32_t)a * (uint32_t)b);
}

struct CombAdd {
  template <class T> __device__ __forceinline__ static T apply(T a, T b) { return comb_add(a, b); }
};
struct CombMul {
  template <class T> __device__ __forceinline__ static T apply(T a, T b) { return comb_mul(a, b); }
};

// ---------------------------------------------------------------- vector loads

// VEC elements of T in one aligned access of VEC*sizeof(T) bytes (4, 8 or 16).
template <class T, int VEC>
struct alignas(sizeof(T) * VEC) Vec {
  T v[VEC];
};

template <class T, int VEC>
__device__ __forceinline__ Vec<T, VEC> load_vec_stream(const T* p) {
  Vec<T, VEC> out;
  constexpr int bytes = sizeof(T) * VEC;
  if constexpr (bytes == 16) {
    uint4 raw = __ldcs(reinterpret_cast<const uint4*>(p));
    out = *reinterpret_cast<Vec<T, VEC>*>(&raw);
  } else if constexpr (bytes == 8) {
    uint2 raw = __ldcs(reinterpret_cast<const uint2*>(p));
    out = *reinterpret_cast<Vec<T, VEC>*>(&raw);
  } else if constexpr (bytes == 4) {
    unsigned int raw = __ldcs(reinterpret_cast<const unsigned int*>(p));
    out = *reinterpret_cast<Vec<T, VEC>*>(&raw);
  } else {
    out = *reinterpret_cast<const Vec<T, VEC>*>(p);
  }
  return out;
}

template <class T, int VEC>
__device__ __forceinline__ Vec<T, VEC> load_vec_cached(const T* p) {
  Vec<T, VEC> out;
  constexpr int bytes = sizeof(T) * VEC;
  if constexpr (bytes == 16) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    out = *reinterpret_cast<Vec<T, VEC>*>(&raw);
  } else if constexpr (bytes == 8) {
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    out = *reinterpret_cast<Vec<T, VEC>*>(&raw);
  } else {
    out = *reinterpret_cast<const Vec<T, VEC>*>(p);
  }
  return out;
}

template <class T, int VEC>
__device__ __forceinline__ void store_vec_stream(T* p, const Vec<T, VEC>& v) {
  constexpr int bytes = sizeof(T) * VEC;
  if constexpr (bytes == 16) {
    __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<const uint4*>(&v));
  } else if constexpr (bytes == 8) {
    __stcs(reinterpret_cast<uint2*>(p), *reinterpret_cast<const uint2*>(&v));
  } else if constexpr (bytes == 4) {
    __stcs(reinterpret_cast<unsigned int*>(p), *reinterpret_cast<const unsigned int*>(&v));
  } else {
    *reinterpret_cast<Vec<T, VEC>*>(p) = v;
  }
}

}  // namespace ppyb200

namespace ppyb200 {

// ---------------------------------------------------------------- async copies to shared

// ---- a warp's ring of row groups in shared memory, filled by bulk copies (the TMA engine:
// one instruction per row group instead of a 16-byte copy per lane and chunk), one mbarrier a
// stage. Measured on the [65536, 1024] f32 row group: 5.58 -> 5.75 TB/s against per-lane
// cp.async copies.
constexpr uint32_t RING_WAIT_LIMIT = 1u << 24;

// lane 0 of the warp: `stages` barriers of one arrival each (the copies add their bytes)
__device__ __forceinline__ void ring_init(uint64_t* bars, int stages) {
  for (int k = 0; k < stages; ++k)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(
        static_cast<unsigned>(__cvta_generic_to_shared(bars + k))));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// one thread: the stage's barrier expects `bytes` (the sum of the copies that follow)
__device__ __forceinline__ void ring_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   static_cast<unsigned>(__cvta_generic_to_shared(bar))),
               "r"(bytes)
               : "memory");
}

// one thread: `bytes` (a multiple of 16) from global `src` to shared `dst`, both 16-byte
// aligned, completing on `bar`. The proxy fence orders the warp's earlier reads of the buffer
// (generic proxy) before the copy's writes (async proxy).
__device__ __forceinline__ void ring_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))),
      "l"(src), "r"(bytes), "r"(static_cast<unsigned>(__cvta_generic_to_shared(bar)))
      : "memory");
}

// every lane: wait (bounded) for the stage's phase of `parity`; on giving up the call's status
// word is raised and the stage is read as it is (in bounds, not the row group)
__device__ __forceinline__ void ring_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
  const unsigned b = static_cast<unsigned>(__cvta_generic_to_shared(bar));
  for (uint32_t tries = 0; tries < RING_WAIT_LIMIT; ++tries) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(b), "r"(parity)
        : "memory");
    if (done) return;
  }
  if (status != nullptr) atomicMax(status, PPYB200_DEVICE_RAISED);
}

// ---- two f32 lanes in one 64-bit register, for the paired FP32 instructions of sm_100
// (add/mul/fma .f32x2: one instruction for two independent f32 operations, each rounded as
// the scalar one would be)
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unf2(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// ---- programmatic dependent launch (sm_90 and later)
//
// A kernel launched with the programmatic-serialization attribute (launch_pdl below) may
// start while the kernel before it on the stream is still running, once every CTA of that
// kernel has run pdl_trigger() or exited: its CTAs then set up (barriers, tensor memory)
// while the previous kernel drains. Such a kernel runs pdl_wait() -- which returns when the
// previous kernel has completed and its memory operations are visible -- before it reads or
// writes any global memory, and every kernel that runs pdl_wait() first has done so
// transitively for all the work before it. A kernel launched without the attribute, or
// after one that never triggers, starts as usual after the previous one completes, and
// pdl_wait() returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- host side

// A value set up once per device for one kernel (its shared-memory attribute, its resident
// cluster count): function attributes and occupancy belong to a device, and one process may
// drive several devices from several threads. `get` runs `setup(int* value)` under a lock the
// first time the calling thread's current device asks, keeps the positive value it gives, and
// hands it back without the lock afterwards. A failed setup is retried by the next call.
struct DeviceOnce {
  static constexpr int kDevices = 64;
  std::mutex lock;
  std::atomic<int> value[kDevices];

  template <class Setup>
  cudaError_t get(Setup&& setup, int* out) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    if (device < 0 || device >= kDevices) return cudaErrorInvalidDevice;
    int v = value[device].load(std::memory_order_acquire);
    if (v <= 0) {
      std::lock_guard<std::mutex> hold(lock);
      v = value[device].load(std::memory_order_relaxed);
      if (v <= 0) {
        e = setup(&v);
        if (e != cudaSuccess) return e;
        if (v <= 0) return cudaErrorInvalidConfiguration;
        value[device].store(v, std::memory_order_release);
      }
    }
    *out = v;
    return cudaSuccess;
  }
};

// Launch `kernel` on `stream` with the programmatic-serialization attribute while
// ppyb200_pdl() is on. The kernel runs pdl_wait() before it touches global memory.
template <class... Params, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = ppyb200_pdl() ? 1 : 0;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

}  // namespace ppyb200
