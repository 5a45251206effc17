// The GPT-2 pieces that are not tensor-dialect groups: the token + position embedding
// gather, the tensor-core linear layers with their epilogues (bias, GELU-tanh, residual
// add), and causal attention. The layernorms come from the backend's row-group code
// (tests/golden/gpt2_layernorm.ppyir built into ppy_b200/prebuilt/gpt2_layernorm).
//
// Layouts: activations row-major [tokens, width] with token t = b * length + l; the residual
// stream in f32, GEMM operands in bf16; weights as torch.nn.Linear keeps them, [out, in]
// (K-major for the tensor cores); the fused QKV projection writes [tokens, 3 * width] with q,
// k, v side by side, head h at columns h * head_dim of each.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "../../include/ppyb200.h"
#include "gemm_sm100.cuh"
#include "gemm_simt.cuh"
#include "ppyb200_device.cuh"

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaStream_t stream_now() { return reinterpret_cast<cudaStream_t>(ppyb200_stream()); }

int32_t finish(cudaError_t error, const char* what, uint64_t launched) {
  if (error != cudaSuccess) return ppyb200_check((int32_t)error, what);
  ppyb200_count_launches(launched);
  return PPYB200_OK;
}

// ---------------------------------------------------------------- embedding

// x[t, c] = wte[ids[t], c] + wpe[t % length, c]: 8 columns per thread, 16-byte loads.
__global__ void __launch_bounds__(256) embed_kernel(const int64_t* __restrict__ ids,
                                                    const __nv_bfloat16* __restrict__ wte,
                                                    const __nv_bfloat16* __restrict__ wpe,
                                                    float* __restrict__ x, int64_t tokens,
                                                    int64_t length, int64_t width,
                                                    int64_t vocab, int32_t* status) {
  const int64_t groups = width / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= tokens * groups) return;
  const int64_t t = i / groups, c = (i % groups) * 8;
  const int64_t id = ids[t];
  if (id < 0 || id >= vocab) {  // an id outside the table: no read, the call raises
    if (status != nullptr) atomicMax(status, PPYB200_DEVICE_RAISED);
    return;
  }
  const uint4 te = __ldg(reinterpret_cast<const uint4*>(wte + id * width + c));
  const uint4 pe = __ldg(reinterpret_cast<const uint4*>(wpe + (t % length) * width + c));
  const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&te);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&pe);
  float4 lo, hi;
  lo.x = __bfloat162float(a[0]) + __bfloat162float(b[0]);
  lo.y = __bfloat162float(a[1]) + __bfloat162float(b[1]);
  lo.z = __bfloat162float(a[2]) + __bfloat162float(b[2]);
  lo.w = __bfloat162float(a[3]) + __bfloat162float(b[3]);
  hi.x = __bfloat162float(a[4]) + __bfloat162float(b[4]);
  hi.y = __bfloat162float(a[5]) + __bfloat162float(b[5]);
  hi.z = __bfloat162float(a[6]) + __bfloat162float(b[6]);
  hi.w = __bfloat162float(a[7]) + __bfloat162float(b[7]);
  float4* dst = reinterpret_cast<float4*>(x + t * width + c);
  dst[0] = lo;
  dst[1] = hi;
}

// ---------------------------------------------------------------- linear epilogues

// tanh on the SFU (PTX tanh.approx.f32, max relative error about 2^-11): the GELU output is
// rounded to bf16 (2^-8) right after, so the approximation does not show in it.
__device__ __forceinline__ float tanh_sfu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh(float z) {
  // 0.5 z (1 + tanh(sqrt(2/pi) (z + 0.044715 z^3))), GPT-2's activation
  const float u = 0.7978845608028654f * (z + 0.044715f * z * z * z);
  return 0.5f * z * (1.0f + tanh_sfu(u));
}

template <int ACTIVATION>  // 0 none, 1 GELU-tanh
struct LinearBf16 {
  const float* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  __device__ __forceinline__ void store_column(const float (&acc)[32], int64_t row0, int64_t col,
                                               int64_t rows) const {
    const float b = bias != nullptr ? __ldg(bias + col) : 0.f;
    __nv_bfloat16* p = out + row0 * ldo + col;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      if (r < rows) {
        float v = acc[r] + b;
        if (ACTIVATION == 1) v = gelu_tanh(v);
        p[r * ldo] = __float2bfloat16_rn(v);
      }
    }
  }
};

struct LinearResidual {
  const float* bias;
  float* residual;  // read and written in place: residual += acc + bias
  int64_t ld;
  __device__ __forceinline__ void store_column(const float (&acc)[32], int64_t row0, int64_t col,
                                               int64_t rows) const {
    const float b = bias != nullptr ? __ldg(bias + col) : 0.f;
    float* p = residual + row0 * ld + col;
    float old[32];
    // all 32 loads first: the rows are independent, their latencies overlap
#pragma unroll
    for (int r = 0; r < 32; ++r) old[r] = r < rows ? p[r * ld] : 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if (r < rows) p[r * ld] = old[r] + (acc[r] + b);
  }
};

// ---------------------------------------------------------------- causal attention

namespace attn {

constexpr int D = 64;     // head dim
constexpr int BQ = 128;   // query rows per CTA (8 warps x 16)
constexpr int BKV = 64;   // keys per tile
constexpr int THREADS = 256;
constexpr int TILE_Q_BYTES = BQ * D * 2;
constexpr int TILE_KV_BYTES = BKV * D * 2;
constexpr int SMEM_BYTES = TILE_Q_BYTES + 4 * TILE_KV_BYTES;  // Q, K[2], V[2]

// byte offset of (row, 8-element chunk) in a [rows][64] bf16 tile: 16-byte chunks XOR-swizzled
// by the row so that 8 consecutive rows of one chunk fall in 8 different bank groups
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Copy `rows` x 64 bf16 (row stride `ld` elements) into a swizzled tile.
__device__ __forceinline__ void load_tile(uint8_t* tile, const __nv_bfloat16* src, int rows,
                                          int64_t ld) {
  for (int i = threadIdx.x; i < rows * 8; i += THREADS) {
    const int row = i >> 3, chunk = i & 7;
    ppyb200::cp_async16(tile + swz(row, chunk), src + row * ld + chunk * 8);
  }
}

// One CTA: 128 query rows of one (batch, head). Warp w owns rows 16w..16w+15; keys stream
// through shared memory in tiles of 64 (double-buffered cp.async), scores and the softmax
// are f32 (online: running max and sum per row), P is rounded to bf16 for the P.V product.
__global__ void __launch_bounds__(THREADS, 2) causal_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                         __nv_bfloat16* __restrict__ out,
                                                         int64_t batch, int64_t length,
                                                         int64_t heads, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sq = smem;
  uint8_t* sk[2] = {smem + TILE_Q_BYTES, smem + TILE_Q_BYTES + TILE_KV_BYTES};
  uint8_t* sv[2] = {smem + TILE_Q_BYTES + 2 * TILE_KV_BYTES,
                    smem + TILE_Q_BYTES + 3 * TILE_KV_BYTES};
  const int64_t q_tiles = length / BQ;
  const int64_t bh_count = batch * heads;
  // the longest (last) query tiles first: they have the most key tiles
  const int64_t qt = q_tiles - 1 - (int64_t)blockIdx.x / bh_count;
  const int64_t bh = (int64_t)blockIdx.x % bh_count;
  const int64_t b = bh / heads, h = bh % heads;
  const int64_t width = heads * D, ld = 3 * width;
  const int64_t q0 = qt * BQ;
  const __nv_bfloat16* base = qkv + (b * length) * ld + h * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const int kv_tiles = (int)((q0 + BQ) / BKV);
  load_tile(sq, base + q0 * ld, BQ, ld);
  load_tile(sk[0], base + width, BKV, ld);
  load_tile(sv[0], base + 2 * width, BKV, ld);
  ppyb200::cp_async_commit();

  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const int64_t q_lo = q0 + warp * 16 + g, q_hi = q_lo + 8;
  const uint32_t sq_u = static_cast<uint32_t>(__cvta_generic_to_shared(sq));

  for (int j = 0; j < kv_tiles; ++j) {
    if (j + 1 < kv_tiles) {
      load_tile(sk[(j + 1) & 1], base + (int64_t)(j + 1) * BKV * ld + width, BKV, ld);
      load_tile(sv[(j + 1) & 1], base + (int64_t)(j + 1) * BKV * ld + 2 * width, BKV, ld);
    }
    ppyb200::cp_async_commit();
    ppyb200::cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int row = warp * 16 + (lane & 15), chunk = ks * 2 + (lane >> 4);
        ldsm_x4(sq_u + swz(row, chunk), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    const uint32_t sk_u = static_cast<uint32_t>(__cvta_generic_to_shared(sk[j & 1]));
    const uint32_t sv_u = static_cast<uint32_t>(__cvta_generic_to_shared(sv[j & 1]));
    // S = Q K^T for this warp's 16 rows and the tile's 64 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int key = p * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int chunk = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sk_u + swz(key, chunk), b0, b1, b2, b3);
        mma16816(s[2 * p], qa[ks], b0, b1);
        mma16816(s[2 * p + 1], qa[ks], b2, b3);
      }
    }
    // scale into log2 units, mask keys after the query, and the online softmax
    const int64_t k0 = (int64_t)j * BKV;
    const bool diagonal = k0 + BKV > q0;
    float mx_lo = m_lo, mx_hi = m_hi;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t key = k0 + nb * 8 + 2 * t + e;
        float lo = s[nb][e] * scale_log2, hi = s[nb][2 + e] * scale_log2;
        if (diagonal) {
          if (key > q_lo) lo = -INFINITY;
          if (key > q_hi) hi = -INFINITY;
        }
        s[nb][e] = lo;
        s[nb][2 + e] = hi;
        mx_lo = fmaxf(mx_lo, lo);
        mx_hi = fmaxf(mx_hi, hi);
      }
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float keep_lo = exp2f(m_lo - mx_lo), keep_hi = exp2f(m_hi - mx_hi);
    m_lo = mx_lo;
    m_hi = mx_hi;
    float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[nb][e] = exp2f(s[nb][e] - m_lo);
        s[nb][2 + e] = exp2f(s[nb][2 + e] - m_hi);
        sum_lo += s[nb][e];
        sum_hi += s[nb][2 + e];
      }
    }
    l_lo = l_lo * keep_lo + sum_lo;
    l_hi = l_hi * keep_hi + sum_hi;
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      o[db][0] *= keep_lo;
      o[db][1] *= keep_lo;
      o[db][2] *= keep_hi;
      o[db][3] *= keep_hi;
    }
    // O += P V: P's accumulator layout is the A operand layout of the next product
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int chunk = p * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sv_u + swz(key, chunk), b0, b1, b2, b3);
        mma16816(o[2 * p], pa, b0, b1);
        mma16816(o[2 * p + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with this tile before it is refilled
  }
  ppyb200::cp_async_wait<0>();
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = 1.f / l_lo, inv_hi = 1.f / l_hi;
  __nv_bfloat16* row_lo = out + (b * length + q_lo) * width + h * D;
  __nv_bfloat16* row_hi = out + (b * length + q_hi) * width + h * D;
#pragma unroll
  for (int db = 0; db < 8; ++db) {
    const int col = db * 8 + 2 * t;
    *reinterpret_cast<uint32_t*>(row_lo + col) = pack_bf16(o[db][0] * inv_lo, o[db][1] * inv_lo);
    *reinterpret_cast<uint32_t*>(row_hi + col) = pack_bf16(o[db][2] * inv_hi, o[db][3] * inv_hi);
  }
}

}  // namespace attn

}  // namespace

extern "C" {

int32_t ppyb200_gpt2_embed(const int64_t* ids, const uint16_t* wte, const uint16_t* wpe,
                           float* x, int64_t tokens, int64_t length, int64_t width,
                           int64_t vocab, int32_t* status) {
  if (tokens <= 0) return PPYB200_OK;
  if (length <= 0 || width % 8 != 0 || !aligned16(wte) || !aligned16(wpe) || !aligned16(x)) {
    ppyb200_set_error("ppyb200_gpt2_embed: width % 8 == 0 and 16-byte aligned tables required");
    return PPYB200_RAISED;
  }
  const int64_t work = tokens * (width / 8);
  embed_kernel<<<(unsigned)((work + 255) / 256), 256, 0, stream_now()>>>(
      ids, reinterpret_cast<const __nv_bfloat16*>(wte), reinterpret_cast<const __nv_bfloat16*>(wpe),
      x, tokens, length, width, vocab, status);
  return finish(cudaGetLastError(), "ppyb200_gpt2_embed", 1);
}

int32_t ppyb200_linear_bf16(const uint16_t* a, const uint16_t* w, const float* bias,
                            uint16_t* out, int64_t m, int64_t n, int64_t k, int32_t activation,
                            int32_t* status) {
  if (m <= 0 || n <= 0) return PPYB200_OK;
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(a);
  const auto* W = reinterpret_cast<const __nv_bfloat16*>(w);
  if (!ppyb200::gemm::tileable(m, n, k) || !aligned16(a) || !aligned16(w) ||
      (activation != 0 && activation != 1)) {
    ppyb200_set_error("ppyb200_linear_bf16: K % 64, 16-byte aligned operands and an "
                      "activation of 0 or 1 required");
    return PPYB200_RAISED;
  }
  auto* O = reinterpret_cast<__nv_bfloat16*>(out);
  cudaError_t e;
  if (activation == 1)
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearBf16<1>{bias, O, n}, status,
                              ppyb200_sm_count(), stream_now());
  else
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearBf16<0>{bias, O, n}, status,
                              ppyb200_sm_count(), stream_now());
  return finish(e, "ppyb200_linear_bf16", 1);
}

int32_t ppyb200_linear_residual(const uint16_t* a, const uint16_t* w, const float* bias,
                                float* residual, int64_t m, int64_t n, int64_t k,
                                int32_t* status) {
  if (m <= 0 || n <= 0) return PPYB200_OK;
  LinearResidual epi{bias, residual, n};
  if (!ppyb200::gemm::tileable(m, n, k) || !aligned16(a) || !aligned16(w)) {
    ppyb200_set_error("ppyb200_linear_residual: K % 64 and 16-byte aligned operands required");
    return PPYB200_RAISED;
  }
  return finish(ppyb200::gemm::launch(reinterpret_cast<const __nv_bfloat16*>(a),
                                      reinterpret_cast<const __nv_bfloat16*>(w), m, n, k, epi,
                                      status, ppyb200_sm_count(), stream_now()),
                "ppyb200_linear_residual", 1);
}

int32_t ppyb200_attention_causal_bf16(const uint16_t* qkv, uint16_t* out, int64_t batch,
                                      int64_t length, int64_t heads, int64_t head_dim) {
  if (batch <= 0 || length <= 0 || heads <= 0) return PPYB200_OK;
  if (head_dim != attn::D || length % attn::BQ != 0 || !aligned16(qkv) || !aligned16(out)) {
    ppyb200_set_error("ppyb200_attention_causal_bf16: head_dim 64, length a multiple of 128 and "
                      "16-byte aligned buffers required");
    return PPYB200_RAISED;
  }
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn::causal_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn::SMEM_BYTES);
    if (e != cudaSuccess) return ppyb200_check((int32_t)e, "attention: shared memory");
    configured = true;
  }
  const int64_t blocks = batch * heads * (length / attn::BQ);
  const float scale_log2 = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  attn::causal_kernel<<<(unsigned)blocks, attn::THREADS, attn::SMEM_BYTES, stream_now()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), reinterpret_cast<__nv_bfloat16*>(out), batch,
      length, heads, scale_log2);
  return finish(cudaGetLastError(), "ppyb200_attention_causal_bf16", 1);
}

}  // extern "C"
