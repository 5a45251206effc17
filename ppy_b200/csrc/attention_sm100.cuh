// Causal attention on Blackwell tensor cores, head_dim 64, bf16 in and out, f32 softmax.
//
// One persistent CTA per SM walks work items (batch, head, pair of 128-query tiles), heaviest
// (last) pairs first, dealt to the CTAs in a snake order (snake_item). The two query tiles of
// a pair share one stream of key tiles (128 keys each); per key tile and query tile t:
//   S_t = Q_t K^T    tcgen05.mma M=128 N=128 K=64 into TMEM (128 columns per query tile)
//   softmax          warpgroup t (4 warps), one query row per thread: tcgen05.ld of its S row,
//                    causal mask on the diagonal tile, P = 2^((S - m) * scale * log2 e) rounded
//                    to bf16 and stored back into TMEM with tcgen05.st (64 columns of bf16
//                    pairs per query tile: the A operand of the next product, which takes it
//                    from TMEM -- no shared-memory round trip), running sum in f32
//   O_t += P V       tcgen05.mma M=128 N=64 K=128, A from TMEM, into TMEM (64 columns per
//                    query tile)
// and at the end O_t / sum goes out as bf16 rows of the merged-heads output. The two
// warpgroups work on their tiles at the same time (two softmax warps per SM sub-partition),
// and the tensor core takes the products of one while the other computes.
//
// The running max m of a row moves only when a new score exceeds it by more than 8 (in units
// of log2): then O and the sum are scaled by 2^(m_old - m_new) (O through tcgen05.ld/st).
// Otherwise the stale m stays, and the probabilities of the tile are at most 2^8 -- exact for
// the result, which divides O by the sum of the same probabilities.
//
//   warps 0-7  softmax (warpgroup t = warps 4t..4t+3; warp w reads TMEM lanes 32 (w % 4)...)
//   warp 8     one thread: TMA loads of the Q tiles (once per item), K and V^T (3-deep ring)
//   warp 9     one thread: the MMAs of query tile 0 and their commits; the warp owns the TMEM
//              allocation
//   warp 10    one thread: the MMAs of query tile 1 (a single issuer serialised the two tiles'
//              waits: 4500 cycles per key tile against about 1500 of tensor-core work)
//   warp 11    idle: it completes the third warpgroup, which gives its registers to the
//              softmax warpgroups (setmaxnreg: 224 a thread for warps 0-7, 56 for 8-11, so
//              that a 128-score row and its state stay in registers)
// Shared-memory operands are all K-major with the 128-byte swizzle: Q and K straight from the
// QKV projection output [tokens, 3 * width]; V from a transposed copy V^T [batch * heads * 64,
// length] that the QKV projection's epilogue writes beside it (keys contiguous).
//
// Every mbarrier wait is bounded as in the matmul kernel: on giving up the CTA raises the call's
// status word, every role leaves its loops, copies and MMAs in flight are drained and the TMEM
// is freed. Every TMA load fills only this CTA's own shared memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "gemm_sm100.cuh"
#include "ppyb200_device.cuh"

namespace ppyb200 {
namespace attention {

using gemm::mbar_arrive;
using gemm::mbar_drain_wait;
using gemm::mbar_expect_tx;
using gemm::mbar_init;
using gemm::mbar_try_wait;
using gemm::smem_desc;
using gemm::smem_u32;
using gemm::tc_fence_after;
using gemm::tc_fence_before;
using gemm::tma_load_2d;

constexpr int D = 64;          // head dim
constexpr int BM = 128;        // queries per query tile
constexpr int BN = 128;        // keys per key tile
constexpr int KV_STAGES = 3;
constexpr int LOADER_WARP = 8, MMA_WARP = 9;
constexpr int THREADS = 384;   // warps 0-7 softmax, 8 loader, 9 and 10 MMA, 11 idle
// Registers per thread after the split (setmaxnreg): the two softmax warpgroups hold a
// 128-score row each and take what the third (one loading thread, two issuing) gives up. The
// launch holds LAUNCH_REGS x 384; the split must not ask for more (launch() checks the
// compiled count before the first launch: an increase the pool cannot meet would never return).
constexpr uint32_t LAUNCH_REGS = 168, SOFTMAX_REGS = 224, SUPPORT_REGS = 56;
static_assert(2 * 128 * SOFTMAX_REGS + 128 * SUPPORT_REGS <= THREADS * LAUNCH_REGS,
              "register split above the launch's registers");
constexpr int Q_BYTES = BM * D * 2;        // [128][64] bf16, one swizzle atom wide
constexpr int K_BYTES = BN * D * 2;        // [128 keys][64 d]
constexpr int V_BYTES = 2 * D * 64 * 2;    // two [64 d][64 keys] halves of V^T
constexpr int TMEM_COLS = 512;             // S_0 [0,128), S_1 [128,256), O_0, O_1 [256,384),
constexpr uint32_t O_COL = 256;            // P_0, P_1 [384,512)
constexpr uint32_t P_COL = 384;            // P_t: 128 bf16 keys a row, two to a column
constexpr uint32_t WAIT_LIMIT = 1u << 22;
constexpr float RESCALE_LOG2 = 8.f;        // the running max moves by more than this, or stays

// kind::f16, bf16 x bf16 -> f32, both K-major: M=128 with N=128 (S) and N=64 (O).
constexpr uint32_t IDESC_S = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(BM >> 4) << 24);
constexpr uint32_t IDESC_O = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(D >> 3) << 17) |
                             ((uint32_t)(BM >> 4) << 24);

struct Shared {
  alignas(1024) uint8_t q[2][Q_BYTES];
  alignas(1024) uint8_t k[KV_STAGES][K_BYTES];
  alignas(1024) uint8_t v[KV_STAGES][V_BYTES];
  alignas(8) uint64_t q_full, q_empty;
  alignas(8) uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  alignas(8) uint64_t s_full[2], s_free[2];
  alignas(8) uint64_t p_full[2];
  alignas(8) uint64_t o_done[2];
  alignas(8) uint64_t drain[2];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void support_registers() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(SUPPORT_REGS));
}
__device__ __forceinline__ void softmax_registers() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(SOFTMAX_REGS));
}

__device__ __forceinline__ bool wait(Shared& s, uint64_t* bar, uint32_t parity, int32_t* status) {
  for (uint32_t tries = 0; tries < WAIT_LIMIT; ++tries) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*(volatile int*)&s.abort) return false;
  }
  *(volatile int*)&s.abort = 1;
  if (status != nullptr) atomicMax(status, PPYB200_DEVICE_RAISED);
  return false;
}

// The softmax warps' wait: every lane waits, and the warp goes on only if all of them saw the
// phase complete (the tcgen05.ld/st after it need the whole warp).
__device__ __forceinline__ bool warp_wait(Shared& s, uint64_t* bar, uint32_t parity,
                                          int32_t* status) {
  const bool ok = wait(s, bar, parity, status);
  return __all_sync(0xffffffffu, ok) != 0;
}

// 2^x on the SFU (PTX ex2.approx.ftz.f32: relative error about 2^-22, 2^-inf = +0); the
// probabilities are rounded to bf16 (2^-8) right after.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

using ppyb200::add2;
using ppyb200::f2;
using ppyb200::fma2;
using ppyb200::unf2;

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                    uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same product with A (M x 16, bf16, K-major) from tensor memory: lane m of `tmem_a` holds
// row m, eight 32-bit columns of two bf16 each (element 2c in the low half of column c).
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 columns of this thread's TMEM lane into v (no wait: tmem_wait_ld() before use)
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// 16 columns of this thread's TMEM lane from w (tcgen05.wait::st before they are read)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* w) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]),
      "r"(w[8]), "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]),
      "r"(w[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Work item i: (batch b, head h, pair p of query tiles 2p and 2p + 1); the heaviest pairs (the
// last, with the most key tiles) first. `has1`: tile 2p + 1 exists (an odd count of query
// tiles leaves the last pair one tile).
struct Item {
  int64_t b, h, p;
  bool has1;
};

__device__ __forceinline__ Item item_of(int64_t i, int64_t bh, int64_t heads, int64_t q_tiles) {
  const int64_t pairs = (q_tiles + 1) / 2;
  Item it;
  it.p = pairs - 1 - i / bh;
  const int64_t r = i % bh;
  it.b = r / heads;
  it.h = r % heads;
  it.has1 = 2 * it.p + 1 < q_tiles;
  return it;
}

// This CTA's item of round `round`: round r covers items [r G, (r + 1) G) of the heaviest-first
// order (G = gridDim.x), CTA c taking the c-th of them in even rounds and the (G - 1 - c)-th in
// odd ones. The CTAs that drew the heaviest items of one round draw the lightest of the next,
// as a longest-first greedy schedule would: with 4 sequences of 1024 tokens (192 items of 15,
// 11, 7 and 3 key tiles for 148 SMs) the busiest CTA walks 15 key tiles instead of 18. Every
// role of the CTA walks the same sequence; an index past the items ends it.
__device__ __forceinline__ int64_t snake_item(int64_t round) {
  const int64_t g = gridDim.x, c = blockIdx.x;
  return round * g + ((round & 1) ? g - 1 - c : c);
}

__global__ void __launch_bounds__(THREADS, 1)
    causal_kernel(const __grid_constant__ CUtensorMap map_qk, const __grid_constant__ CUtensorMap map_vt,
                  __nv_bfloat16* __restrict__ out, int64_t batch, int64_t length, int64_t heads,
                  float scale_log2, int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  Shared& s = *reinterpret_cast<Shared*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q_tiles = length / BM;
  const int64_t bh = batch * heads;
  const int64_t items = bh * ((q_tiles + 1) / 2);
  const int64_t width = heads * D;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 2);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_free[i], 4);
      mbar_init(&s.p_full[i], 4);
      mbar_init(&s.o_done[i], 1);
    }
    mbar_init(&s.drain[0], 1);
    mbar_init(&s.drain[1], 1);
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // the set-up above overlaps the previous kernel; its results are needed from here on
  pdl_wait();
  pdl_trigger();
  // Each role takes its share of the register split first, with the whole warp (the four
  // warps of a warpgroup ask for the same count).
  if (warp == LOADER_WARP) {
    support_registers();
    if (lane == 0) {
      // ---- loader
      uint64_t kv = 0, qi = 0;
      bool ok = true;
      int64_t round = 0;
      for (int64_t i = snake_item(0); i < items && ok; i = snake_item(++round), ++qi) {
        const Item it = item_of(i, bh, heads, q_tiles);
        const int32_t row0 = (int32_t)(it.b * length);
        const int q_count = it.has1 ? 2 : 1;
        if (!wait(s, &s.q_empty, (uint32_t)((qi & 1) ^ 1), status)) break;
        mbar_expect_tx(&s.q_full, (uint32_t)(q_count * Q_BYTES));
        for (int t = 0; t < q_count; ++t)
          tma_load_2d(s.q[t], &map_qk, &s.q_full, (int32_t)(it.h * D),
                      row0 + (int32_t)((2 * it.p + t) * BM));
        const int64_t tiles = 2 * it.p + q_count;
        for (int64_t j = 0; j < tiles; ++j, ++kv) {
          const int st = (int)(kv % KV_STAGES);
          if (!wait(s, &s.kv_empty[st], (uint32_t)(((kv / KV_STAGES) & 1) ^ 1), status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&s.kv_full[st], K_BYTES + V_BYTES);
          tma_load_2d(s.k[st], &map_qk, &s.kv_full[st], (int32_t)(width + it.h * D),
                      row0 + (int32_t)(j * BN));
          const int32_t vrow = (int32_t)((it.b * heads + it.h) * D);
          tma_load_2d(s.v[st], &map_vt, &s.kv_full[st], (int32_t)(j * BN), vrow);
          tma_load_2d(s.v[st] + V_BYTES / 2, &map_vt, &s.kv_full[st], (int32_t)(j * BN + 64),
                      vrow);
        }
      }
      // the copies issued here land before the CTA may leave
      const uint64_t first = kv > (uint64_t)KV_STAGES ? kv - KV_STAGES : 0;
      for (uint64_t j = first; j < kv; ++j)
        mbar_drain_wait(&s.kv_full[j % KV_STAGES], (uint32_t)((j / KV_STAGES) & 1));
      if (qi > 0) mbar_drain_wait(&s.q_full, (uint32_t)((qi - 1) & 1));
    }
  } else if (warp == MMA_WARP || warp == MMA_WARP + 1) {
    support_registers();
    if (lane == 0) {
      // ---- MMA issuers: warp MMA_WARP + t issues the products of query tile t, so that one
      // tile's waits never hold up the other's products. Step j: S_t(j), then
      // O_t += P_t(j-1) V(j-1). tcgen05.commit tracks the products of the committing thread,
      // so the stage and Q barriers take one arrival from each issuer: a commit after its
      // products, or a plain arrival for a key tile (or a Q tile) it has no product of --
      // given only after waiting for that stage's (that Q's) load, so that the arrival falls
      // in the phase it belongs to.
      const int t = warp - MMA_WARP;
      uint64_t kv = 0, qi = 0, sc = 0, pc = 0;  // S and PV products issued for this tile
      bool ok = true;
      int64_t round = 0;
      for (int64_t i = snake_item(0); i < items && ok; i = snake_item(++round), ++qi) {
        const Item it = item_of(i, bh, heads, q_tiles);
        const int64_t tiles = it.has1 ? 2 * it.p + 2 : 2 * it.p + 1;  // key tiles loaded
        const int64_t mine = t == 0 ? 2 * it.p + 1 : (it.has1 ? 2 * it.p + 2 : 0);
        if (!wait(s, &s.q_full, (uint32_t)(qi & 1), status)) break;
        tc_fence_after();
        if (mine == 0) mbar_arrive(&s.q_empty);
        for (int64_t j = 0; j <= tiles && ok; ++j) {
          if (j < mine) {
            const uint64_t kj = kv + (uint64_t)j;
            const int st = (int)(kj % KV_STAGES);
            if (!wait(s, &s.kv_full[st], (uint32_t)((kj / KV_STAGES) & 1), status) ||
                !wait(s, &s.s_free[t], (uint32_t)((sc & 1) ^ 1), status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t kdesc = smem_desc(s.k[st]);
            const uint64_t qdesc = smem_desc(s.q[t]);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma(tmem + (uint32_t)(t * BN), qdesc + (uint64_t)(kk * 2),
                  kdesc + (uint64_t)(kk * 2), IDESC_S, kk > 0 ? 1u : 0u);
            commit(&s.s_full[t]);
            ++sc;
            if (j == mine - 1) commit(&s.q_empty);
          }
          if (j >= 1) {
            const int64_t jp = j - 1;
            const uint64_t kj = kv + (uint64_t)jp;
            const int st = (int)(kj % KV_STAGES);
            if (jp < mine) {
              if (!wait(s, &s.p_full[t], (uint32_t)(pc & 1), status)) {
                ok = false;
                break;
              }
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < BN / 16; ++kk) {
                const int half = kk >> 2, off = (kk & 3) * 2;
                const uint64_t vdesc = smem_desc(s.v[st] + half * (V_BYTES / 2)) + (uint64_t)off;
                mma_ts(tmem + O_COL + (uint32_t)(t * D), tmem + P_COL + (uint32_t)(t * 64 + kk * 8),
                       vdesc, IDESC_O, (jp > 0 || kk > 0) ? 1u : 0u);
              }
              commit(&s.o_done[t]);
              ++pc;
              commit(&s.kv_empty[st]);
            } else if (jp < tiles) {
              if (!wait(s, &s.kv_full[st], (uint32_t)((kj / KV_STAGES) & 1), status)) {
                ok = false;
                break;
              }
              mbar_arrive(&s.kv_empty[st]);
            }
          }
        }
        kv += (uint64_t)tiles;
      }
      commit(&s.drain[t]);
      mbar_drain_wait(&s.drain[t], 0);
    }
  } else if (warp > MMA_WARP + 1) {
    support_registers();  // the idle warp of the third warpgroup
  } else {
    softmax_registers();
    // ---- softmax: warpgroup t = warp / 4 takes query tile 2p + t; thread = query row. The
    // running max m is kept in raw score units.
    const int t = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + (uint32_t)(t * BN);
    const uint32_t o_addr = tmem + lane_addr + O_COL + (uint32_t)(t * D);
    const uint32_t p_addr = tmem + lane_addr + P_COL + (uint32_t)(t * 64);
    const uint64_t scale2 = f2(scale_log2, scale_log2);
    uint64_t sc = 0, pc = 0;
    bool ok = true;
    int64_t round = 0;
    for (int64_t i = snake_item(0); i < items && ok; i = snake_item(++round)) {
      const Item it = item_of(i, bh, heads, q_tiles);
      if (t == 1 && !it.has1) continue;
      const int64_t qt = 2 * it.p + t;
      const int64_t tiles = qt + 1;
      float m = -INFINITY, l = 0.f;
      for (int64_t j = 0; j < tiles; ++j) {
        if (!warp_wait(s, &s.s_full[t], (uint32_t)(sc & 1), status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_ld32_nowait(s_addr + (uint32_t)(c * 32), sv + c * 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.s_free[t]);
        ++sc;
        if (j == tiles - 1) {
          // the diagonal tile (key tile j = query tile qt): keys after the query are masked
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c > row) sv[c] = -INFINITY;
        }
        float mx[4] = {m, m, m, m};
#pragma unroll
        for (int c = 0; c < BN; c += 8) {
          mx[0] = max3(mx[0], sv[c + 0], sv[c + 1]);
          mx[1] = max3(mx[1], sv[c + 2], sv[c + 3]);
          mx[2] = max3(mx[2], sv[c + 4], sv[c + 5]);
          mx[3] = max3(mx[3], sv[c + 6], sv[c + 7]);
        }
        const float m_tile = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        // move the running max only by more than RESCALE_LOG2 (m = -inf on the first tile)
        const bool move = (m_tile - m) * scale_log2 > RESCALE_LOG2;
        float alpha = 1.f;
        if (move) {
          alpha = ex2((m - m_tile) * scale_log2);  // 0 on the first tile
          m = m_tile;
          l *= alpha;
        }
        const float shift = -m * scale_log2;
        const uint64_t shift2 = f2(shift, shift);
        // P_t(j-1) was read by the previous product into O_t, which the rescale below
        // rewrites: P_t(j) and the rescale wait for that product
        if (pc > 0) {
          if (!warp_wait(s, &s.o_done[t], (uint32_t)((pc - 1) & 1), status)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int quarter = 0; quarter < 4; ++quarter) {
          // 32 probabilities, packed to bf16 pairs and stored as they are made (the scores
          // they replace free their registers)
          uint32_t pk[16];
#pragma unroll
          for (int c = quarter * 32; c < quarter * 32 + 32; c += 2) {
            float lo, hi;
            unf2(fma2(f2(sv[c], sv[c + 1]), scale2, shift2), lo, hi);
            const float e0 = ex2(lo), e1 = ex2(hi);
            sum2[(c >> 1) & 3] = add2(sum2[(c >> 1) & 3], f2(e0, e1));
            pk[(c >> 1) & 15] = pack(e0, e1);
          }
          tmem_st16(p_addr + (uint32_t)(quarter * 16), pk);
        }
        float s0, s1, s2, s3;
        unf2(add2(sum2[0], sum2[1]), s0, s1);
        unf2(add2(sum2[2], sum2[3]), s2, s3);
        l += (s0 + s1) + (s2 + s3);
        if (j > 0 && __any_sync(0xffffffffu, move)) {
          // some rows' max moved: scale those rows of O_t (the previous products' sum)
          float o[D];
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            tmem_ld32_nowait(o_addr + (uint32_t)(c * 32), o + c * 32);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < D; ++e) o[e] *= alpha;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) tmem_st32(o_addr + (uint32_t)(c * 32), o + c * 32);
          tmem_wait_st();
        }
        // P in tensor memory becomes the A operand of O_t += P V once its stores completed
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.p_full[t]);
        ++pc;
      }
      if (!ok) break;
      // O_t / l for this row, as bf16, once the tile's last product has completed
      if (!warp_wait(s, &s.o_done[t], (uint32_t)((pc - 1) & 1), status)) break;
      tc_fence_after();
      const float inv = 1.f / l;
      float o[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32_nowait(o_addr + (uint32_t)(c * 32), o + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __nv_bfloat16* dst = out + (it.b * length + qt * BM + row) * width + it.h * D;
#pragma unroll
      for (int e = 0; e < D; e += 8) {
        uint4 packed;
        packed.x = pack(o[e + 0] * inv, o[e + 1] * inv);
        packed.y = pack(o[e + 2] * inv, o[e + 3] * inv);
        packed.z = pack(o[e + 4] * inv, o[e + 5] * inv);
        packed.w = pack(o[e + 6] * inv, o[e + 7] * inv);
        *reinterpret_cast<uint4*>(dst + e) = packed;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
  }
}

inline size_t shared_bytes() { return sizeof(Shared) + 1024; }

// A row-major [rows, cols] bf16 matrix as a TMA map of [box_rows, 64] tiles, 128-byte swizzle.
inline bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                     int64_t row_stride, int box_rows) {
  gemm::EncodeTiled encode = gemm::encode_tiled();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 2)};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// What the kernel takes: head_dim 64, length a whole number of 128-query tiles, extents whose
// rows and columns fit the TMA maps (int32 coordinates).
inline bool tileable(int64_t batch, int64_t length, int64_t heads, int64_t head_dim) {
  return batch > 0 && heads > 0 && head_dim == D && length > 0 && length % BM == 0 &&
         batch * length < (1ll << 31) && batch * heads * D < (1ll << 31) &&
         3 * heads * D < (1ll << 31);
}

// Launch on `stream`: qkv [batch*length, 3*heads*64] (q and k columns read), vt
// [batch*heads*64, length] (V transposed per head), out [batch*length, heads*64]. The caller
// checks `tileable` and 16-byte alignment of the three buffers.
inline cudaError_t launch(const __nv_bfloat16* qkv, const __nv_bfloat16* vt, __nv_bfloat16* out,
                          int64_t batch, int64_t length, int64_t heads, int32_t* status,
                          int sm_count, cudaStream_t stream) {
  const int64_t width = heads * D;
  CUtensorMap map_qk, map_vt;
  if (!make_map(&map_qk, qkv, batch * length, 3 * width, 3 * width, BM) ||
      !make_map(&map_vt, vt, batch * heads * D, length, length, D))
    return cudaErrorInvalidValue;
  static gemm::DeviceOnce configured;
  int ready = 0;
  cudaError_t e = configured.get(
      [](int* v) {
        cudaFuncAttributes attributes;
        cudaError_t r = cudaFuncGetAttributes(&attributes, causal_kernel);
        if (r != cudaSuccess) return r;
        // the register split needs the launch's full LAUNCH_REGS a thread
        *v = attributes.numRegs == (int)LAUNCH_REGS ? 1 : 0;
        return cudaFuncSetAttribute(causal_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)shared_bytes());
      },
      &ready);
  if (e != cudaSuccess) return e;
  if (ready != 1) return cudaErrorInvalidKernelImage;
  const int64_t items = batch * heads * ((length / BM + 1) / 2);
  const int grid = (int)(items < sm_count ? items : sm_count);
  const float scale_log2 = 0.125f * 1.4426950408889634f;  // log2(e) / sqrt(64)
  return launch_pdl(causal_kernel, dim3(grid), dim3(THREADS), shared_bytes(), stream, map_qk,
                    map_vt, out, batch, length, heads, scale_log2, status);
}

}  // namespace attention
}  // namespace ppyb200
