// Dense matmul on Blackwell tensor cores: D[M,N] = A[M,K] @ Bt[N,K]^T accumulated in f32,
// then an elementwise epilogue that stores it, for bf16 A and Bt (both K-major: a row-major
// A and a row-major [N,K] B^T -- the layout torch.nn.Linear keeps its weight in). K must be
// a multiple of 64; M and N may be ragged (TMA fills the out-of-range part of an edge tile
// with zeros and the epilogue skips it).
//
// One persistent CTA per SM walks the output tiles (128 x 256) in L2-friendly bands:
//   warp 0   one thread issues TMA loads of A and Bt tiles (K-step 64, 128-byte swizzle)
//            into a STAGES-deep shared-memory ring;
//   warp 1   one thread issues tcgen05.mma (M=128, N=256, K=16) into a TMEM accumulator
//            and commits each stage back to the loader; it also owns the TMEM allocation;
//   warps 2-9 read the accumulator out of TMEM (tcgen05.ld; warp w reads lane quarter w % 4,
//            two warps per quarter split the columns), apply the epilogue and store rows
//            of C coalesced through shared memory.
// The accumulator is double-buffered (2 x 256 TMEM columns), so the epilogue of one tile
// runs while the MMAs of the next are issued.
//
// Every mbarrier wait is bounded: past its limit the waiting thread records
// PPYB200_DEVICE_RAISED in the call's status word and raises the CTA's abort flag; every
// role then leaves its loop, the loader waits (bounded) for the copies it issued, the MMA
// thread waits (bounded) for its MMAs, and the TMEM is freed before the CTA exits.
// Every TMA load fills only this CTA's own shared memory (the kernel may run on several GPUs
// of one node).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

#include "ppyb200_device.cuh"
#include "../../include/ppyb200.h"

namespace ppyb200 {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;  // tile width; 192 where N is a multiple of 192 (pick_tile_n)
constexpr int BK = 64;  // 64 bf16 = 128 bytes: one swizzle row
constexpr int UMMA_K = 16;
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr int A_BYTES = BM * BK * 2;
// two accumulators of up to BN f32 columns (at columns 0 and TBN of the allocation)
constexpr int TMEM_COLS = 2 * BN;
constexpr int EPI_PITCH = 33;       // floats per staged row (32 + 1 pad: no bank conflicts)
constexpr int EPI_BYTES = EPI_WARPS * 32 * EPI_PITCH * 4;
constexpr int GROUP_M = 16;         // tiles walk bands of 16 M-blocks for L2 reuse
constexpr uint32_t WAIT_LIMIT = 1u << 22;


// What a kernel's operands are. Every K-step loads one 128-byte swizzle row of each operand
// row (64 bf16 or 32 f32) and issues four MMAs of 32 bytes of K each (K = 16 bf16, or K = 8
// tf32), so the shared-memory layouts, descriptors and the ring are the same for both; what
// differs is the element type of the TMA maps, the MMA kind, and which columns of the operand
// matrices a K-step reads.
//
// Bf16Operands: A [M, K] and Bt [N, K], bf16; K-step kb reads columns kb*64 .. +63 of both.
struct Bf16Operands {
  using T = __nv_bfloat16;
  static constexpr int kStep = 64;
  static constexpr int kSegments = 1;
  static constexpr bool kChunked = false;  // one accumulation per tile, over all of K
  static constexpr uint32_t kFormat = 1;  // bf16 (kind::f16)
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  // The columns of A and Bt the K-steps of a tile read, in order: kb * 64 for both.
  struct Walk {
    int64_t kb = 0;
    __device__ __forceinline__ Walk(int64_t, int64_t) {}
    __device__ __forceinline__ void restart() { kb = 0; }
    __device__ __forceinline__ int32_t a_col() const { return (int32_t)(kb * kStep); }
    __device__ __forceinline__ int32_t b_col() const { return (int32_t)(kb * kStep); }
    __device__ __forceinline__ void next() { ++kb; }
  };
};

// Tf32x3Operands: an f32 product A.B computed as three tf32 products on the tensor cores,
// A_hi.B_hi + A_hi.B_lo + A_lo.B_hi, where x_hi is x rounded to tf32 (11 significant bits)
// and x_lo is (x - x_hi) rounded to tf32: what is dropped is A_lo.B_lo and the third
// 11-bit piece of each operand, both about 2^-22 of |a||b| (fp32 keeps 24 bits). The
// operands are A2 [M, 2 Kp] = [A_hi | A_lo] and B2t [N, 2 Kp] = [B_hi^T | B_lo^T] (Kp = K
// rounded up to 32, zero-filled), written by the split in gemm_f32.cuh.
//
// The tensor core adds each MMA's products into the f32 accumulator with a truncation whose
// errors do not cancel: over n MMAs they grow like n * 2^-24 of the sum (measured: 1.5e-4 of
// the rms at K = 4096 when the three products ran back to back, the small ones added last to
// the full-size sum). So K is walked in chunks of cs 32-wide steps (cs = the largest divisor
// of Kp/32 up to 8: 256 columns): each chunk's A_lo.B_hi, then A_hi.B_lo, then A_hi.B_hi go
// into a fresh accumulator -- the small products first, while the sum is small -- and the
// epilogue warps add the chunks' sums up in registers with f32 adds. K-step kb of a tile is
// step r = kb % (3 cs) of chunk q = kb / (3 cs): part p = r / cs (0: A_lo.B_hi, 1: A_hi.B_lo,
// 2: A_hi.B_hi) at 32-wide column j = q cs + r % cs of K (Walk keeps these as counters).
struct Tf32x3Operands {
  using T = float;
  static constexpr int kStep = 32;
  static constexpr int kSegments = 3;
  static constexpr bool kChunked = true;
  static constexpr uint32_t kFormat = 2;  // tf32 (kind::tf32)
  static constexpr CUtensorMapDataType kMapType = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  // K-steps per chunk of each product, for `per` 32-wide steps in all
  __host__ __device__ __forceinline__ static int64_t chunk_steps(int64_t per) {
    int64_t cs = per < 8 ? per : 8;
    while (per % cs != 0) --cs;
    return cs;
  }
  // The columns of A2 and B2t the K-steps of a tile read, in order, kept as counters
  // (chunk q, part p, step jj within the part) so that a step costs no division.
  struct Walk {
    int64_t per, cs, q = 0, jj = 0;
    int p = 0;
    __device__ __forceinline__ Walk(int64_t per_, int64_t cs_) : per(per_), cs(cs_) {}
    __device__ __forceinline__ void restart() {
      q = 0;
      jj = 0;
      p = 0;
    }
    __device__ __forceinline__ int32_t a_col() const {
      const int64_t j = q * cs + jj;
      return (int32_t)((p == 0 ? per + j : j) * kStep);
    }
    __device__ __forceinline__ int32_t b_col() const {
      const int64_t j = q * cs + jj;
      return (int32_t)((p == 1 ? per + j : j) * kStep);
    }
    __device__ __forceinline__ void next() {
      if (++jj == cs) {
        jj = 0;
        if (++p == 3) {
          p = 0;
          ++q;
        }
      }
    }
  };
};


// The instruction descriptor of an M x TBN product with f32 accumulation for operands `Op`,
// both K-major (PTX ISA, tcgen05 instruction descriptor: c_format bits 4-5, a/b format bits
// 7-12, N>>3 at bit 17, M>>4 at bit 24).
template <class Op, int TBN = BN>
constexpr uint32_t idesc(int m) {
  return (1u << 4) | (Op::kFormat << 7) | (Op::kFormat << 10) | ((uint32_t)(TBN >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// The one-CTA kernel's shared memory for tiles TBN columns wide (256, or 192 for N a multiple
// of 192: see pick_tile_n).
template <int TBN>
struct SharedT {
  static constexpr int kStageBytes = A_BYTES + TBN * BK * 2;
  // the operand ring, 1024-byte aligned for the 128-byte swizzle
  alignas(1024) uint8_t stage[STAGES][kStageBytes];
  float epi[EPI_WARPS][32][EPI_PITCH];
  alignas(8) uint64_t full[STAGES];
  alignas(8) uint64_t empty[STAGES];
  alignas(8) uint64_t acc_full[2];
  alignas(8) uint64_t acc_empty[2];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase of `parity` to complete, at most WAIT_LIMIT tries; on giving up (or
// when another role already gave up) raise the abort flag and the status word.
template <class Layout>
__device__ __forceinline__ bool mbar_wait(Layout& s, uint64_t* bar, uint32_t parity,
                                          int32_t* status) {
  for (uint32_t tries = 0; tries < WAIT_LIMIT; ++tries) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*(volatile int*)&s.abort) return false;
  }
  *(volatile int*)&s.abort = 1;
  if (status != nullptr) atomicMax(status, PPYB200_DEVICE_RAISED);
  return false;
}

// A bounded wait used while tearing down: it ignores the abort flag.
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t tries = 0; tries < WAIT_LIMIT; ++tries)
    if (mbar_try_wait(bar, parity)) return;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with the 128-byte swizzle: start
// address (>>4) at bit 0, leading offset 16 B (unused for this layout) at bit 16, 1024 B
// between 8-row groups at bit 32, descriptor version 1 at bit 46, swizzle mode 2 at bit 61.
__device__ __forceinline__ uint64_t smem_desc(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// One M=128 x N=TBN MMA of 32 bytes of K from the operand tiles at adesc, bdesc.
template <class Op, int TBN>
__device__ __forceinline__ void mma_step(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
  if constexpr (Op::kFormat == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc<Op, TBN>(BM)), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc<Op, TBN>(BM)), "r"(accumulate));
  }
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.ld without the wait: the 32 registers are not to be read before tmem_ld_wait(r),
// which takes them as in/out operands so that every use of them is ordered after it.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
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
}

__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
                 "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]),
                 "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tile_coords(int64_t t, int64_t m_blocks, int64_t n_blocks,
                                            int64_t& mb, int64_t& nb) {
  const int64_t per_group = (int64_t)GROUP_M * n_blocks;
  const int64_t group = t / per_group;
  const int64_t first_m = group * GROUP_M;
  const int64_t rows = (m_blocks - first_m) < GROUP_M ? (m_blocks - first_m) : GROUP_M;
  const int64_t r = t % per_group;
  mb = first_m + r % rows;
  nb = r / rows;
}

// The epilogue: `__device__ void store(float acc, int64_t row, int64_t col) const` is called
// once per element of C inside [0, M) x [0, N); consecutive lanes get consecutive columns of
// one row, so stores through it coalesce. This one writes acc (+ bias[col]) as f32.
//
// The kernel hands an epilogue 32 rows of one column at a time:
// `store_column(const float (&acc)[32], int64_t row0, int64_t col, int64_t rows)` stores
// acc[r] at (row0 + r, col) for r < rows. `for_column` gives that from a per-element store.
// (Every loop over the 32 values is unrolled in full: an index the compiler cannot resolve
// would put the array in local memory.)
// An epilogue may instead take whole rows: with `static constexpr bool kRows = true` the kernel
// calls `store_row(const float (&acc)[32], int64_t row, int64_t col0, int64_t cols)` with acc[j]
// at (row, col0 + j) for j < cols (cols = 32 except at a ragged right edge): the values a lane
// reads from tensor memory, with no transpose, for epilogues whose rows it can write as 16-byte
// vectors.
//
// Or it may take four consecutive columns of eight rows at a time: with
// `static constexpr bool kQuads = true` the kernel calls
// `store_quads(const float4 (&v)[8], int64_t row, int count, int64_t col)` with v[i] the four
// values at (row + 4 i, col..col+3) for i < count (col % 4 == 0; all inside C when N % 4 == 0),
// after turning the 32 x 32 block through shared memory so that eight lanes cover one row's
// 128 bytes: every 16-byte access of the warp then covers four whole 128-byte rows. For f32
// outputs whose rows start on 16-byte boundaries.
template <class E, class = void>
struct takes_rows : std::false_type {};
template <class E>
struct takes_rows<E, std::void_t<decltype(E::kRows)>> : std::integral_constant<bool, E::kRows> {};
template <class E, class = void>
struct takes_quads : std::false_type {};
template <class E>
struct takes_quads<E, std::void_t<decltype(E::kQuads)>> : std::integral_constant<bool, E::kQuads> {};
// Or, for bf16 C whose rows start on 16-byte boundaries and N % 64 == 0, it may hand over whole
// 128-byte lines: with `static constexpr bool kLines = true`, members `__nv_bfloat16* out` and
// `int64_t ldo`, and `pack32(const float (&acc)[32], int64_t col0, uint32_t (&pk)[16])` giving
// the bf16 pairs of 32 columns of one row (bias and activation applied), the kernel takes two
// adjacent 32-column chunks at a time -- 64 bf16, one line of each row --, turns the 32 rows'
// lines through shared memory (16-byte slots XOR-swizzled by the row) and stores them eight
// lanes per line: each 16-byte store instruction of the warp writes four whole lines, where
// the row form writes 16 bytes into each of 32 rows and leaves every sector it touches half
// written until its next instruction.
template <class E, class = void>
struct takes_lines : std::false_type {};
template <class E>
struct takes_lines<E, std::void_t<decltype(E::kLines)>> : std::integral_constant<bool, E::kLines> {};
// A kLines epilogue may also have `bool is_line(int64_t col)`: where it is false, the pair of
// chunks from `col` goes to its `store_row` (the row form) instead.
template <class E, class = void>
struct has_is_line : std::false_type {};
template <class E>
struct has_is_line<E, std::void_t<decltype(std::declval<const E&>().is_line(int64_t{}))>>
    : std::true_type {};

template <class Epi>
__device__ __forceinline__ void for_column(const Epi& epi, const float (&acc)[32], int64_t row0,
                                           int64_t col, int64_t rows) {
#pragma unroll
  for (int r = 0; r < 32; ++r)
    if (r < rows) epi.store(acc[r], row0 + r, col);
}

struct BiasEpilogue {
  const float* bias;
  float* c;
  int64_t ldc;
  __device__ __forceinline__ void store(float acc, int64_t row, int64_t col) const {
    __stcs(c + row * ldc + col, bias != nullptr ? acc + __ldg(bias + col) : acc);
  }
  __device__ __forceinline__ void store_column(const float (&acc)[32], int64_t row0, int64_t col,
                                               int64_t rows) const {
    for_column(*this, acc, row0, col, rows);
  }
};

// C = A.B + bias by four-column quads: eight lanes store one row's 32 consecutive floats as
// float4s, four rows per instruction, so rows that start on 128-byte lines take whole lines
// at a quarter of the column form's store instructions. c and bias 16-byte aligned, ldc % 4
// == 0; a quad that crosses N stores its columns below N one at a time.
struct BiasQuads {
  static constexpr bool kQuads = true;
  const float* bias;
  float* c;
  int64_t ldc;
  int64_t n;
  __device__ __forceinline__ void store_quads(const float4 (&v)[8], int64_t row, int count,
                                              int64_t col) const {
    float* p = c + row * ldc + col;
    if (col + 4 <= n) {
      const float4 b = bias != nullptr ? __ldg(reinterpret_cast<const float4*>(bias + col))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < count)
          __stcs(reinterpret_cast<float4*>(p + 4 * i * ldc),
                 make_float4(v[i].x + b.x, v[i].y + b.y, v[i].z + b.z, v[i].w + b.w));
      return;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i >= count) break;
      const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      for (int j = 0; j < 4 && col + j < n; ++j)
        __stcs(p + 4 * i * ldc + j, bias != nullptr ? e[j] + __ldg(bias + col + j) : e[j]);
    }
  }
};


// The chunked form's epilogue pieces. A warp's share of a tile is 32 rows (its lane
// quarter) x TBN/2 columns (its half), held as sum[c][j] = column 32 c + j of the lane's row.
template <int TBN>
__device__ __forceinline__ void add_chunk(float (&sum)[TBN / 64][32], uint32_t acc, int half) {
#pragma unroll
  for (int c = 0; c < TBN / 64; ++c) {
    uint32_t r[32];
    tmem_ld32(acc + (uint32_t)((half * (TBN / 64) + c) * 32), r);
#pragma unroll
    for (int j = 0; j < 32; ++j) sum[c][j] += __uint_as_float(r[j]);
  }
}

// Hand the summed share to the epilogue's store_column, one column of 32 rows per lane
// (turned through the warp's staging rows, as epilogue_tile's column form).
template <int TBN, class Epi>
__device__ __forceinline__ void store_sum(const Epi& epi, float (*stage_rows)[EPI_PITCH],
                                          const float (&sum)[TBN / 64][32], int half, int lane,
                                          int64_t row0, int64_t col0, int64_t rows,
                                          int64_t n) {
#pragma unroll
  for (int c = 0; c < TBN / 64; ++c) {
#pragma unroll
    for (int j = 0; j < 32; ++j) stage_rows[lane][j] = sum[c][j];
    __syncwarp();
    const int64_t col = col0 + (half * (TBN / 64) + c) * 32 + lane;
    if (col < n && rows > 0) {
      float column[32];
#pragma unroll
      for (int rr = 0; rr < 32; ++rr) column[rr] = stage_rows[rr][lane];
      epi.store_column(column, row0, col, rows);
    }
    __syncwarp();
  }
}

// One accumulator tile's epilogue for one warp: the 32 rows of its lane quarter (from row0,
// `rows` of them inside C), the half of the TBN columns from col0 + half * TBN / 2; `acc` is the
// TMEM address of the quarter's lanes at the accumulator's first column.
template <int TBN, class Epi>
__device__ __forceinline__ void epilogue_tile(const Epi& epi, float (*stage_rows)[EPI_PITCH],
                                              uint32_t acc, int half, int lane, int64_t row0,
                                              int64_t col0, int64_t rows, int64_t n) {
  // The warp's half is NC chunks of 32 columns, taken as a stream: the TMEM load of chunk
  // c + 1 is in flight while chunk c is turned and stored (one 32-column load ahead; the
  // loads were one round trip each, back to back with the stores, in a warp that is one of
  // two on its sub-partition).
  // An epilogue that mixes line and row stores (QKV's v columns) keeps the load just before
  // each chunk: its registers do not hold a second chunk without spilling.
  constexpr int NC = TBN / 64;
  constexpr bool ahead = !has_is_line<Epi>::value;
  const int base = half * NC;
  uint32_t r[32], next[32];
  uint32_t pk0[16];  // the lines form: the first chunk of a pair, packed
  if constexpr (ahead) {
    tmem_ld32_async(acc + (uint32_t)(base * 32), r);
    tmem_ld_wait(r);
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int chunk = base + c;
    if constexpr (ahead) {
      if (c + 1 < NC) tmem_ld32_async(acc + (uint32_t)((chunk + 1) * 32), next);
    } else {
      tmem_ld32_async(acc + (uint32_t)(chunk * 32), r);
      tmem_ld_wait(r);
    }
    if constexpr (takes_lines<Epi>::value) {
      static_assert(NC % 2 == 0, "the lines form takes pairs of 32-column chunks per half");
      uint4* line = reinterpret_cast<uint4*>(&stage_rows[0][0]);  // 32 rows x 8 slots of 16 B
      const int64_t col = col0 + (chunk & ~1) * 32;  // the line's first column (N % 64 == 0)
      bool as_line = true;
      if constexpr (has_is_line<Epi>::value) {
        as_line = epi.is_line(col);  // the same for the whole warp: it depends on col alone
        if (!as_line) {
          const int64_t cc = col0 + chunk * 32;
          if (lane < rows && cc < n) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            epi.store_row(v, row0 + lane, cc, n - cc < 32 ? n - cc : 32);
          }
        }
      }
      if (!as_line) {
        // stored by rows above
      } else if ((c & 1) == 0) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (col < n) epi.pack32(v, col, pk0);
      } else {
        uint32_t pk1[16];
        {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (col < n) epi.pack32(v, col + 32, pk1);
        }
        const int slot = lane & 7;
        if (col < n) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            line[lane * 8 + (q ^ (lane & 7))] =
                make_uint4(pk0[4 * q], pk0[4 * q + 1], pk0[4 * q + 2], pk0[4 * q + 3]);
            line[lane * 8 + ((q + 4) ^ (lane & 7))] =
                make_uint4(pk1[4 * q], pk1[4 * q + 1], pk1[4 * q + 2], pk1[4 * q + 3]);
          }
        }
        __syncwarp();
        if (col < n) {
          uint4 v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = (lane >> 3) + 4 * i;
            v[i] = line[rr * 8 + (slot ^ (rr & 7))];
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = (lane >> 3) + 4 * i;
            if (rr < rows)
              *reinterpret_cast<uint4*>(epi.out + (row0 + rr) * epi.ldo + col + 8 * slot) = v[i];
          }
        }
        __syncwarp();
      }
    } else if constexpr (takes_rows<Epi>::value) {
      // lane holds row (row0 + lane), columns chunk*32 .. +31, as the epilogue takes them
      const int64_t col = col0 + chunk * 32;
      if (lane < rows && col < n) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        epi.store_row(v, row0 + lane, col, n - col < 32 ? n - col : 32);
      }
    } else if constexpr (takes_quads<Epi>::value) {
      // 32 rows x 8 float4 in shared memory, the float4 slot XOR-swizzled by the row so that
      // both the row-wise writes and the column-wise reads are free of bank conflicts
      float4* quad = reinterpret_cast<float4*>(&stage_rows[0][0]);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        quad[lane * 8 + (q ^ (lane & 7))] =
            make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                        __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
      __syncwarp();
      const int64_t col = col0 + chunk * 32 + 4 * (lane & 7);
      float4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = (lane >> 3) + 4 * i;
        v[i] = quad[rr * 8 + ((lane & 7) ^ (rr & 7))];
      }
      __syncwarp();
      // rows (lane >> 3) + 4 i inside C: i < (rows - (lane >> 3) + 3) / 4
      const int count = rows > (lane >> 3) ? (int)((rows - (lane >> 3) + 3) / 4) : 0;
      if (col < n && count > 0) epi.store_quads(v, row0 + (lane >> 3), count < 8 ? count : 8, col);
    } else {
      // lane holds row (row0 + lane), columns chunk*32 .. +31: turn it through shared
      // memory so that lane j then holds column chunk*32 + j of all 32 rows
#pragma unroll
      for (int j = 0; j < 32; ++j) stage_rows[lane][j] = __uint_as_float(r[j]);
      __syncwarp();
      const int64_t col = col0 + chunk * 32 + lane;
      if (col < n && rows > 0) {
        float column[32];
#pragma unroll
        for (int rr = 0; rr < 32; ++rr) column[rr] = stage_rows[rr][lane];
        epi.store_column(column, row0, col, rows);
      }
      __syncwarp();
    }
    if constexpr (ahead) {
      if (c + 1 < NC) {
        tmem_ld_wait(next);
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = next[j];
      }
    }
  }
}

// The one-CTA kernel's body, for operands `Op`; `k` is the columns of one operand segment
// (K for bf16, Kp for tf32x3), a multiple of Op::kStep.
template <class Op, int TBN, class Epi>
__device__ __forceinline__ void matmul_single_body(const CUtensorMap& map_a,
                                                   const CUtensorMap& map_b, int64_t m,
                                                   int64_t n, int64_t k, const Epi& epi,
                                                   int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  SharedT<TBN>& s = *reinterpret_cast<SharedT<TBN>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t per = k / Op::kStep;  // K-steps per operand segment
  const int64_t m_blocks = (m + BM - 1) / BM, n_blocks = (n + TBN - 1) / TBN;
  const int64_t k_blocks = Op::kSegments * per;
  const int64_t tiles = m_blocks * n_blocks;
  // K-steps that share one accumulator: the whole tile, or one chunk (Tf32x3Operands)
  int64_t cs = 0, group = k_blocks;
  if constexpr (Op::kChunked) {
    cs = Op::chunk_steps(per);
    group = 3 * cs;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], EPI_WARPS);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
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

  if (warp == 0) {
    if (lane == 0) {
      // ---- loader
      uint64_t it = 0;
      bool ok = true;
      typename Op::Walk walk(per, cs);
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int64_t mb, nb;
        tile_coords(t, m_blocks, n_blocks, mb, nb);
        walk.restart();
        for (int64_t kb = 0; kb < k_blocks; ++kb, ++it, walk.next()) {
          const int st = (int)(it % STAGES);
          const uint32_t phase = (uint32_t)((it / STAGES) & 1);
          if (!mbar_wait(s, &s.empty[st], phase ^ 1, status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&s.full[st], SharedT<TBN>::kStageBytes);
          tma_load_2d(s.stage[st], &map_a, &s.full[st], walk.a_col(), (int32_t)(mb * BM));
          tma_load_2d(s.stage[st] + A_BYTES, &map_b, &s.full[st], walk.b_col(),
                      (int32_t)(nb * TBN));
        }
      }
      // the copies this thread issued land before the CTA may leave
      const uint64_t first = it > (uint64_t)STAGES ? it - STAGES : 0;
      for (uint64_t j = first; j < it; ++j)
        mbar_drain_wait(&s.full[j % STAGES], (uint32_t)((j / STAGES) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: one accumulator buffer per `group` K-steps (acc_it counts them)
      uint64_t it = 0, acc_it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        uint32_t d = 0;
        int64_t r = 0;  // K-step within the group
        for (int64_t kb = 0; kb < k_blocks; ++kb, ++it) {
          const int a = (int)(acc_it & 1);
          if (r == 0) {
            const uint32_t aphase = (uint32_t)((acc_it >> 1) & 1);
            if (!mbar_wait(s, &s.acc_empty[a], aphase ^ 1, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            d = tmem + (uint32_t)(a * TBN);
          }
          const int st = (int)(it % STAGES);
          const uint32_t phase = (uint32_t)((it / STAGES) & 1);
          if (!mbar_wait(s, &s.full[st], phase, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc(s.stage[st]);
          const uint64_t bdesc = smem_desc(s.stage[st] + A_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // advancing K by 32 bytes inside the swizzle row: +2 in addr >> 4
            mma_step<Op, TBN>(d, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2),
                         (r > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&s.empty[st]);
          if (++r == group) {
            mma_commit(&s.acc_full[a]);
            ++acc_it;
            r = 0;
          }
        }
      }
      // every MMA issued has finished before the accumulator memory is freed
      mma_commit(&s.drain);
      mbar_drain_wait(&s.drain, 0);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32); the two warps of a
    // quarter take alternate halves of the 256 columns
    const int quarter = warp & 3;
    const int ew = warp - 2;
    const int half = ew >> 2;
    float(*stage_rows)[EPI_PITCH] = s.epi[ew];
    uint64_t acc_it = 0;
    if constexpr (Op::kChunked) {
      // each chunk's accumulator added into registers, the tile stored after the last
      const int64_t chunks = k_blocks / group;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        float sum[TBN / 64][32];
#pragma unroll
        for (int c = 0; c < TBN / 64; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[c][j] = 0.f;
        for (int64_t q = 0; q < chunks; ++q, ++acc_it) {
          const int a = (int)(acc_it & 1);
          const uint32_t aphase = (uint32_t)((acc_it >> 1) & 1);
          if (!mbar_wait(s, &s.acc_full[a], aphase, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          add_chunk<TBN>(sum, tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * TBN),
                    half);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.acc_empty[a]);
        }
        if (!ok) break;
        int64_t mb, nb;
        tile_coords(t, m_blocks, n_blocks, mb, nb);
        const int64_t row0 = mb * BM + quarter * 32;
        const int64_t rows = m - row0 < 32 ? m - row0 : 32;
        store_sum<TBN>(epi, stage_rows, sum, half, lane, row0, nb * TBN, rows, n);
      }
    } else {
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++acc_it) {
        const int a = (int)(acc_it & 1);
        const uint32_t aphase = (uint32_t)((acc_it >> 1) & 1);
        if (!mbar_wait(s, &s.acc_full[a], aphase, status)) break;
        tc_fence_after();
        int64_t mb, nb;
        tile_coords(t, m_blocks, n_blocks, mb, nb);
        const int64_t row0 = mb * BM + quarter * 32;
        const int64_t col0 = nb * TBN;
        const int64_t rows = m - row0 < 32 ? m - row0 : 32;
        epilogue_tile<TBN>(epi, stage_rows,
                      tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * TBN), half,
                      lane, row0, col0, rows, n);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.acc_empty[a]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
  }
}

template <class Epi, int TBN = BN>
__global__ void __launch_bounds__(THREADS, 1)
    matmul_bf16_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, int64_t m, int64_t n,
                       int64_t k, Epi epi, int32_t* status) {
  matmul_single_body<Bf16Operands, TBN>(map_a, map_b, m, n, k, epi, status);
}

template <class Epi, int TBN = BN>
__global__ void __launch_bounds__(THREADS, 1)
    matmul_tf32x3_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b, int64_t m, int64_t n,
                         int64_t k, Epi epi, int32_t* status) {
  matmul_single_body<Tf32x3Operands, TBN>(map_a, map_b, m, n, k, epi, status);
}

// ---- the 2-CTA form: a cluster of two CTAs on two SMs computes 256 x 256 tiles with
// tcgen05.mma.cta_group::2 (M = 256: each CTA holds 128 rows of A and 128 rows of B^T in its
// shared memory and 128 rows of the accumulator in its TMEM). Per CTA a K-step moves 32 KB
// instead of 48 KB for the same 128 x 256 x 64 of work: the operand bytes that bound the
// one-CTA kernel at small K shrink by a third.
//   both CTAs' warp 0   TMA loads of their halves, completing on the first CTA's `full`
//                       barrier (the cta_group::2 form of the load; no multicast)
//   first CTA's warp 1  the MMAs; each commit arrives on the barrier in both CTAs
//   both CTAs' warps 2-9  the epilogue of their own 128 rows; they release the accumulator
//                       on the first CTA's `acc_empty`
// Every wait is bounded as in the one-CTA kernel; the two CTAs meet at cluster barriers only
// before and after their loops, which every path leaves.
constexpr int PAIR_STAGES = 5;

template <int TBN>
struct PairSharedT {
  static constexpr int kStageBytes = A_BYTES + (TBN / 2) * BK * 2;  // each CTA's half of B
  alignas(1024) uint8_t stage[PAIR_STAGES][kStageBytes];
  float epi[EPI_WARPS][32][EPI_PITCH];
  alignas(8) uint64_t full[PAIR_STAGES];
  alignas(8) uint64_t empty[PAIR_STAGES];
  alignas(8) uint64_t acc_full[2];
  alignas(8) uint64_t acc_empty[2];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of the variable at `addr` in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// One M=256 x N=TBN MMA of 32 bytes of K over the pair (issued by the first CTA).
template <class Op, int TBN>
__device__ __forceinline__ void mma_pair_step(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t accumulate) {
  if constexpr (Op::kFormat == 2) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc<Op, TBN>(2 * BM)), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc<Op, TBN>(2 * BM)), "r"(accumulate));
  }
}

// Arrive on `bar` (same offset) in both CTAs of the pair once this thread's MMAs are done.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// Arrive on a barrier of either CTA of the pair (a shared::cluster address). The arrive only
// tells the MMA warp that this warp's tcgen05.ld reads of an accumulator are done (ordered by
// tcgen05.wait::ld and tcgen05.fence::before_thread_sync before it), so it keeps the default
// CTA-scope release: a cluster-scope release would first wait for every global store the warp
// has in flight (the tile's output) to become visible to the cluster, which measured as
// 2.8 cycles of membar stall per issued instruction in the GPT-2 LM head.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// The 2-CTA kernel's body, for operands `Op` (`k` as for matmul_single_body).
template <class Op, int TBN, class Epi>
__device__ __forceinline__ void matmul_pair_body(const CUtensorMap& map_a,
                                                 const CUtensorMap& map_b, int64_t m,
                                                 int64_t n, int64_t k, const Epi& epi,
                                                 int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  PairSharedT<TBN>& s = *reinterpret_cast<PairSharedT<TBN>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool first = rank == 0;
  const int64_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int64_t m_blocks = (m + 2 * BM - 1) / (2 * BM), n_blocks = (n + TBN - 1) / TBN;
  const int64_t per = k / Op::kStep;  // K-steps per operand segment
  const int64_t k_blocks = Op::kSegments * per, tiles = m_blocks * n_blocks;
  // K-steps that share one accumulator: the whole tile, or one chunk (Tf32x3Operands)
  int64_t cs = 0, group = k_blocks;
  if constexpr (Op::kChunked) {
    cs = Op::chunk_steps(per);
    group = 3 * cs;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < PAIR_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 2 * EPI_WARPS);  // both CTAs' epilogue warps
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    // both CTAs, the same warp: one allocation spanning the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the barriers of both CTAs exist before any load or commit reaches them
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // the set-up above overlaps the previous kernel; its results are needed from here on
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- loader (both CTAs): this CTA's 128 rows of A and of B^T
      uint64_t it = 0;
      bool ok = true;
      typename Op::Walk walk(per, cs);
      for (int64_t t = pair; t < tiles && ok; t += pairs) {
        int64_t mb, nb;
        tile_coords(t, m_blocks, n_blocks, mb, nb);
        walk.restart();
        for (int64_t kb = 0; kb < k_blocks; ++kb, ++it, walk.next()) {
          const int st = (int)(it % PAIR_STAGES);
          const uint32_t phase = (uint32_t)((it / PAIR_STAGES) & 1);
          if (!mbar_wait(s, &s.empty[st], phase ^ 1, status)) {
            ok = false;
            break;
          }
          if (first) mbar_expect_tx(&s.full[st], 2 * PairSharedT<TBN>::kStageBytes);
          const uint32_t bar = mapa_shared(smem_u32(&s.full[st]), 0);
          tma_load_2d_pair(s.stage[st], &map_a, bar, walk.a_col(),
                           (int32_t)(mb * 2 * BM + rank * BM));
          tma_load_2d_pair(s.stage[st] + A_BYTES, &map_b, bar, walk.b_col(),
                           (int32_t)(nb * TBN + rank * (TBN / 2)));
        }
      }
      // the pair's copies land before the CTAs may leave (they all complete on the first
      // CTA's barriers; the second CTA leaves only after the cluster barrier below)
      if (first) {
        const uint64_t from = it > (uint64_t)PAIR_STAGES ? it - PAIR_STAGES : 0;
        for (uint64_t j = from; j < it; ++j)
          mbar_drain_wait(&s.full[j % PAIR_STAGES], (uint32_t)((j / PAIR_STAGES) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      if (first) {
        // ---- MMA issuer (first CTA): one accumulator buffer per `group` K-steps
        uint64_t it = 0, acc_it = 0;
        bool ok = true;
        for (int64_t t = pair; t < tiles && ok; t += pairs) {
          uint32_t d = 0;
          int64_t r = 0;  // K-step within the group
          for (int64_t kb = 0; kb < k_blocks; ++kb, ++it) {
            const int a = (int)(acc_it & 1);
            if (r == 0) {
              const uint32_t aphase = (uint32_t)((acc_it >> 1) & 1);
              if (!mbar_wait(s, &s.acc_empty[a], aphase ^ 1, status)) {
                ok = false;
                break;
              }
              tc_fence_after();
              d = tmem + (uint32_t)(a * TBN);
            }
            const int st = (int)(it % PAIR_STAGES);
            const uint32_t phase = (uint32_t)((it / PAIR_STAGES) & 1);
            if (!mbar_wait(s, &s.full[st], phase, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t adesc = smem_desc(s.stage[st]);
            const uint64_t bdesc = smem_desc(s.stage[st] + A_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / UMMA_K; ++kk)
              mma_pair_step<Op, TBN>(d, adesc + (uint64_t)(kk * 2), bdesc + (uint64_t)(kk * 2),
                                (r > 0 || kk > 0) ? 1u : 0u);
            mma_commit_pair(&s.empty[st]);
            if (++r == group) {
              mma_commit_pair(&s.acc_full[a]);
              ++acc_it;
              r = 0;
            }
          }
        }
        mma_commit_pair(&s.drain);
      }
      // every MMA writing this CTA's TMEM has finished before it is freed
      mbar_drain_wait(&s.drain, 0);
    }
  } else {
    // ---- epilogue (both CTAs): this CTA's 128 rows of each 256 x 256 tile
    const int quarter = warp & 3;
    const int ew = warp - 2;
    const int half = ew >> 2;
    float(*stage_rows)[EPI_PITCH] = s.epi[ew];
    uint64_t acc_it = 0;
    if constexpr (Op::kChunked) {
      // each chunk's accumulator added into registers, the tile stored after the last
      const int64_t chunks = k_blocks / group;
      bool ok = true;
      for (int64_t t = pair; t < tiles && ok; t += pairs) {
        float sum[TBN / 64][32];
#pragma unroll
        for (int c = 0; c < TBN / 64; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[c][j] = 0.f;
        for (int64_t q = 0; q < chunks; ++q, ++acc_it) {
          const int a = (int)(acc_it & 1);
          const uint32_t aphase = (uint32_t)((acc_it >> 1) & 1);
          if (!mbar_wait(s, &s.acc_full[a], aphase, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          add_chunk<TBN>(sum, tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * TBN),
                    half);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&s.acc_empty[a]), 0));
        }
        if (!ok) break;
        int64_t mb, nb;
        tile_coords(t, m_blocks, n_blocks, mb, nb);
        const int64_t row0 = mb * 2 * BM + rank * BM + quarter * 32;
        const int64_t rows = m - row0 < 32 ? m - row0 : 32;
        store_sum<TBN>(epi, stage_rows, sum, half, lane, row0, nb * TBN, rows, n);
      }
    } else {
      for (int64_t t = pair; t < tiles; t += pairs, ++acc_it) {
        const int a = (int)(acc_it & 1);
        const uint32_t aphase = (uint32_t)((acc_it >> 1) & 1);
        if (!mbar_wait(s, &s.acc_full[a], aphase, status)) break;
        tc_fence_after();
        int64_t mb, nb;
        tile_coords(t, m_blocks, n_blocks, mb, nb);
        const int64_t row0 = mb * 2 * BM + rank * BM + quarter * 32;
        const int64_t col0 = nb * TBN;
        const int64_t rows = m - row0 < 32 ? m - row0 : 32;
        epilogue_tile<TBN>(epi, stage_rows,
                      tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * TBN), half,
                      lane, row0, col0, rows, n);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&s.acc_empty[a]), 0));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs are done with the pair's TMEM and barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
  }
}

template <class Epi, int TBN = BN>
__global__ void __launch_bounds__(THREADS, 1)
    matmul_bf16_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                            const __grid_constant__ CUtensorMap map_b, int64_t m, int64_t n,
                            int64_t k, Epi epi, int32_t* status) {
  matmul_pair_body<Bf16Operands, TBN>(map_a, map_b, m, n, k, epi, status);
}

template <class Epi, int TBN = BN>
__global__ void __launch_bounds__(THREADS, 1)
    matmul_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                              const __grid_constant__ CUtensorMap map_b, int64_t m, int64_t n,
                              int64_t k, Epi epi, int32_t* status) {
  matmul_pair_body<Tf32x3Operands, TBN>(map_a, map_b, m, n, k, epi, status);
}

// ---- host side

using ppyb200::DeviceOnce;

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled lookup_encode_tiled() {
  void* entry = nullptr;
  cudaDriverEntryPointQueryResult found;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &entry, cudaEnableDefault, &found) ==
          cudaSuccess &&
      found == cudaDriverEntryPointSuccess)
    return reinterpret_cast<EncodeTiled>(entry);
  return nullptr;
}

// The driver's tensor-map encoder (the same function for every device), looked up once.
inline EncodeTiled encode_tiled() {
  static const EncodeTiled fn = lookup_encode_tiled();
  return fn;
}

// A row-major [rows, cols] matrix of Op::T as a TMA map of [box_rows, Op::kStep] tiles (one
// 128-byte swizzle row wide), 128-byte swizzle.
template <class Op>
inline bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                     int box_rows) {
  EncodeTiled encode = encode_tiled();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * (int64_t)sizeof(typename Op::T))};
  const cuuint32_t box[2] = {(cuuint32_t)Op::kStep, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, Op::kMapType, 2, const_cast<void*>(base), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// What the tensor-core kernel takes: K a whole number of 64-wide steps (the row stride of A
// and Bt, K * 2 bytes, is then a multiple of 16 as TMA requires), extents within int32.
inline bool tileable(int64_t m, int64_t n, int64_t k) {
  return m > 0 && n > 0 && k > 0 && k % BK == 0 && k < (1ll << 31) && m < (1ll << 31) &&
         n < (1ll << 31);
}

template <int TBN = BN>
inline size_t shared_bytes() { return sizeof(SharedT<TBN>) + 1024; }

// The __global__ kernels of operands `Op` with epilogue `Epi`, tiles TBN columns wide.
template <class Op, class Epi, int TBN>
struct Kernels;
template <class Epi, int TBN>
struct Kernels<Bf16Operands, Epi, TBN> {
  static constexpr auto single = matmul_bf16_kernel<Epi, TBN>;
  static constexpr auto pair = matmul_bf16_pair_kernel<Epi, TBN>;
};
template <class Epi, int TBN>
struct Kernels<Tf32x3Operands, Epi, TBN> {
  static constexpr auto single = matmul_tf32x3_kernel<Epi, TBN>;
  static constexpr auto pair = matmul_tf32x3_pair_kernel<Epi, TBN>;
};

// The one-CTA kernel on `stream` over operand matrices a [m, Op::kSegments > 1 ? 2k : k] and
// bt [n, same] (see the operand structs); returns a cudaError_t (cudaErrorInvalidValue when
// the maps cannot be made). The caller checks the shapes and 16-byte alignment of a, bt.
template <class Op, int TBN = BN, class Epi>
inline cudaError_t launch_single_op(const typename Op::T* a, const typename Op::T* bt, int64_t m,
                                    int64_t n, int64_t k, Epi epi, int32_t* status, int sm_count,
                                    cudaStream_t stream) {
  const int64_t cols = Op::kSegments > 1 ? 2 * k : k;
  CUtensorMap map_a, map_b;
  if (!make_map<Op>(&map_a, a, m, cols, BM) || !make_map<Op>(&map_b, bt, n, cols, TBN))
    return cudaErrorInvalidValue;
  static DeviceOnce configured;
  int ready = 0;
  cudaError_t e = configured.get(
      [](int* v) {
        *v = 1;
        return cudaFuncSetAttribute(Kernels<Op, Epi, TBN>::single,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)shared_bytes<TBN>());
      },
      &ready);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((m + BM - 1) / BM) * ((n + TBN - 1) / TBN);
  const int grid = (int)(tiles < sm_count ? tiles : sm_count);
  return launch_pdl(Kernels<Op, Epi, TBN>::single, dim3(grid), dim3(THREADS),
                    shared_bytes<TBN>(), stream, map_a, map_b, m, n, k, epi, status);
}

template <int TBN = BN>
inline size_t pair_shared_bytes() { return sizeof(PairSharedT<TBN>) + 1024; }

// K from which a tile's MMAs, not its stores, set its pace (C = A.B + bias keeps the column
// form there: quads measured 2.5 % slower at 8192^3, and faster at K = 768).
constexpr int64_t DEEP_K = 2048;


// The 2-CTA kernel on `stream`: clusters of two CTAs, as many as can be resident at once (at
// most one per 256 x 256 tile). Same contract as `launch_single_op`.
template <class Op, int TBN = BN, class Epi>
inline cudaError_t launch_pair_op(const typename Op::T* a, const typename Op::T* bt, int64_t m,
                                  int64_t n, int64_t k, Epi epi, int32_t* status,
                                  cudaStream_t stream) {
  const int64_t cols = Op::kSegments > 1 ? 2 * k : k;
  CUtensorMap map_a, map_b;
  if (!make_map<Op>(&map_a, a, m, cols, BM) || !make_map<Op>(&map_b, bt, n, cols, TBN / 2))
    return cudaErrorInvalidValue;
  static DeviceOnce resident;
  cudaLaunchConfig_t config = {};
  cudaLaunchAttribute attribute[2];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = 2;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[1].val.programmaticStreamSerializationAllowed = 1;
  config.blockDim = dim3(THREADS, 1, 1);
  config.dynamicSmemBytes = pair_shared_bytes<TBN>();
  config.stream = stream;
  config.attrs = attribute;
  config.numAttrs = 1;
  // the clusters of two CTAs that fit on this device at once (after the shared-memory
  // attribute that lets the kernel launch at all)
  int max_clusters = 0;
  cudaError_t e = resident.get(
      [&config](int* v) {
        cudaError_t r = cudaFuncSetAttribute(Kernels<Op, Epi, TBN>::pair,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)pair_shared_bytes<TBN>());
        if (r != cudaSuccess) return r;
        cudaLaunchConfig_t probe = config;
        probe.gridDim = dim3(2, 1, 1);
        return cudaOccupancyMaxActiveClusters(v, Kernels<Op, Epi, TBN>::pair, &probe);
      },
      &max_clusters);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((m + 2 * BM - 1) / (2 * BM)) * ((n + TBN - 1) / TBN);
  const int64_t clusters = tiles < max_clusters ? tiles : max_clusters;
  config.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  config.numAttrs = ppyb200_pdl() ? 2 : 1;
  return cudaLaunchKernelEx(&config, Kernels<Op, Epi, TBN>::pair, map_a, map_b, m, n, k, epi,
                            status);
}

template <class Epi>
inline cudaError_t launch_single(const __nv_bfloat16* a, const __nv_bfloat16* bt, int64_t m,
                                 int64_t n, int64_t k, Epi epi, int32_t* status, int sm_count,
                                 cudaStream_t stream) {
  return launch_single_op<Bf16Operands>(a, bt, m, n, k, epi, status, sm_count, stream);
}

// The tile width for an m x n x k product on `units` SMs (one CTA per tile) or CTA pairs, in
// rows of `block_rows`: 192 when n is a whole number of 192-wide tiles and fewer waves x width
// are needed than with 256 -- GPT-2's out projection (N = 768, K = 768): 0.744 against 0.793
// ms per forward at 32768 rows (7 waves of 192 against 6 of 256 on 74 CTA pairs). At deep K a
// 192-wide tile loads a third more operand bytes per MMA than a 256-wide one and the loads set
// the pace when several waves run (the proj layer, K = 3072, took 2.09 against 1.79 ms at
// 32768 rows), so there 192 is taken only when the 256-wide tiles do not fill one wave: the
// proj layer at 4096 rows (48 of 74 pairs busy with 256, 64 with 192). Else 256.
inline int pick_tile_n(int64_t m, int64_t n, int64_t k, int64_t block_rows, int64_t units) {
  if (n % 192 != 0 || units < 1) return BN;
  const int64_t rows = (m + block_rows - 1) / block_rows;
  const int64_t wide = rows * ((n + 255) / 256), narrow = rows * (n / 192);
  if (k >= DEEP_K && (wide >= units || narrow > units)) return BN;
  const int64_t cost_wide = (wide + units - 1) / units * 256;
  const int64_t cost_narrow = (narrow + units - 1) / units * 192;
  return cost_narrow < cost_wide ? 192 : BN;
}

// The tensor-core GEMM: CTA pairs or one CTA per tile, as ppyb200_gemm_form() says (by shape
// by default), over bf16 A [m, k] and Bt [n, k]. Same contract as `launch_single_op`.
template <class Epi>
inline cudaError_t launch(const __nv_bfloat16* a, const __nv_bfloat16* bt, int64_t m, int64_t n,
                          int64_t k, Epi epi, int32_t* status, int sm_count,
                          cudaStream_t stream) {
  const int32_t form = ppyb200_gemm_form();
  // By shape: CTA pairs from two row blocks up. They halve each SM's operand loads and, with
  // the accumulator released at CTA scope, measured faster than one CTA per tile at every
  // GPT-2 shape (32768 rows, K = 768: out projection 0.765 against 0.829 ms, QKV 1.32 against
  // 1.35, FC 1.92 against 1.95 per forward; K = 3072 and 8192: 3 % and 2.4 %). Below 256
  // rows half of each pair would idle.
  const bool pairs = form == PPYB200_GEMM_PAIRS || (form == PPYB200_GEMM_BY_SHAPE && m >= 2 * BM);
  // the 192-wide tile for the epilogue forms that take it (not whole 128-byte lines of
  // pairs of 32-column chunks); ppyb200_gemm_form pins 256 with its PAIRS / SINGLE values
  if constexpr (!takes_lines<Epi>::value) {
    if (form == PPYB200_GEMM_BY_SHAPE &&
        pick_tile_n(m, n, k, pairs ? 2 * BM : BM, pairs ? sm_count / 2 : sm_count) == 192) {
      if (pairs) return launch_pair_op<Bf16Operands, 192>(a, bt, m, n, k, epi, status, stream);
      return launch_single_op<Bf16Operands, 192>(a, bt, m, n, k, epi, status, sm_count, stream);
    }
  }
  if (pairs) return launch_pair_op<Bf16Operands>(a, bt, m, n, k, epi, status, stream);
  return launch_single_op<Bf16Operands>(a, bt, m, n, k, epi, status, sm_count, stream);
}

}  // namespace gemm
}  // namespace ppyb200
