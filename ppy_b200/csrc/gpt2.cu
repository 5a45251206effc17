// The GPT-2 pieces that are not tensor-dialect groups: the token + position embedding
// gather, the tensor-core linear layers with their epilogues (bias, GELU-tanh, residual
// add), and causal attention. The layernorms come from the backend's row-group code
// (tests/golden/gpt2_layernorm.ppyir built into ppy_b200/prebuilt/gpt2_layernorm).
//
// Layouts: activations row-major [tokens, width] with token t = b * length + l; the residual
// stream in f32, GEMM operands in bf16; weights as torch.nn.Linear keeps them, [out, in]
// (K-major for the tensor cores); the fused QKV projection writes q and k into
// [tokens, 3 * width] (q, k, v side by side, head h at columns h * head_dim of each) and v
// transposed per head into [batch * heads * head_dim, length], the layouts the tensor-core
// attention kernel reads (attention_sm100.cuh).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "../../include/ppyb200.h"
#include "attention_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_simt.cuh"
#include "ppyb200_device.cuh"

namespace {

using ppyb200::add2;
using ppyb200::f2;
using ppyb200::fma2;
using ppyb200::mul2;
using ppyb200::unf2;

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
  ppyb200::pdl_wait();  // the previous kernel may still read x
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

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// GELU-tanh of two values in one 64-bit register, packed to bf16x2 (see LinearBf16Lines).
__device__ __forceinline__ uint32_t gelu_pair(uint64_t z) {
  const uint64_t k1 = f2(0.7978845608028654f, 0.7978845608028654f);
  const uint64_t k2 = f2(0.7978845608028654f * 0.044715f, 0.7978845608028654f * 0.044715f);
  const uint64_t halves = f2(0.5f, 0.5f);
  const uint64_t u = mul2(z, fma2(mul2(z, z), k2, k1));
  float u0, u1;
  unf2(u, u0, u1);
  const uint64_t t = f2(tanh_sfu(u0), tanh_sfu(u1));
  const uint64_t h = mul2(z, halves);
  float g0, g1;
  unf2(fma2(h, t, h), g0, g1);
  return pack_bf16x2(g0, g1);
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

// Row and four-column forms of the epilogues above (gemm_sm100.cuh), for outputs whose rows
// start on 16-byte boundaries: 16-byte loads and stores.
__device__ __forceinline__ void load_bias32(const float* bias, int64_t col0, float (&b)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 v = bias != nullptr ? __ldg(reinterpret_cast<const float4*>(bias + col0) + q)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    b[4 * q] = v.x;
    b[4 * q + 1] = v.y;
    b[4 * q + 2] = v.z;
    b[4 * q + 3] = v.w;
  }
}


template <int ACTIVATION>
struct LinearBf16Rows {  // ldo % 8 == 0, out and bias 16-byte aligned
  static constexpr bool kRows = true;
  const float* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  __device__ __forceinline__ void store_row(const float (&acc)[32], int64_t row, int64_t col0,
                                            int64_t cols) const {
    __nv_bfloat16* p = out + row * ldo + col0;
    if (cols == 32) {
      float b[32];
      load_bias32(bias, col0, b);
      uint32_t pk[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float v0 = acc[2 * k] + b[2 * k], v1 = acc[2 * k + 1] + b[2 * k + 1];
        if (ACTIVATION == 1) {
          v0 = gelu_tanh(v0);
          v1 = gelu_tanh(v1);
        }
        pk[k] = pack_bf16x2(v0, v1);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<uint4*>(p)[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                                                    pk[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < cols) {
          float v = acc[j] + (bias != nullptr ? __ldg(bias + col0 + j) : 0.f);
          if (ACTIVATION == 1) v = gelu_tanh(v);
          p[j] = __float2bfloat16_rn(v);
        }
      }
    }
  }
};

// The same bf16 outputs handed to the kernel as whole 128-byte lines (the kLines form):
// N % 64 == 0, ldo % 8 == 0, out and bias 16-byte aligned.
template <int ACTIVATION>
struct LinearBf16Lines {
  static constexpr bool kLines = true;
  const float* bias;
  __nv_bfloat16* out;
  int64_t ldo;
  // Two columns at a time on the paired FP32 instructions: z = acc + bias, and for GELU-tanh
  // u = z (k1 + k2 z^2) (k1 = sqrt(2/pi), k2 = 0.044715 k1: the same polynomial as
  // gelu_tanh, regrouped), t = tanh(u), 0.5 z (1 + t) = h + h t with h = z / 2 -- five
  // paired instructions and two tanh per pair instead of eleven scalar ones.
  __device__ __forceinline__ void pack32(const float (&acc)[32], int64_t col0,
                                         uint32_t (&pk)[16]) const {
    const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = bias != nullptr ? __ldg(b4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      const uint64_t z01 = add2(f2(acc[4 * q], acc[4 * q + 1]), f2(b.x, b.y));
      const uint64_t z23 = add2(f2(acc[4 * q + 2], acc[4 * q + 3]), f2(b.z, b.w));
      if (ACTIVATION == 1) {
        pk[2 * q] = gelu_pair(z01);
        pk[2 * q + 1] = gelu_pair(z23);
      } else {
        float lo, hi;
        unf2(z01, lo, hi);
        pk[2 * q] = pack_bf16x2(lo, hi);
        unf2(z23, lo, hi);
        pk[2 * q + 1] = pack_bf16x2(lo, hi);
      }
    }
  }
};

struct LinearResidualQuads {  // ld % 4 == 0, N % 4 == 0, residual and bias 16-byte aligned
  static constexpr bool kQuads = true;
  const float* bias;
  float* residual;
  int64_t ld;
  __device__ __forceinline__ void store_quads(const float4 (&v)[8], int64_t row, int count,
                                              int64_t col) const {
    const float4 b = bias != nullptr ? __ldg(reinterpret_cast<const float4*>(bias + col))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    float* p = residual + row * ld + col;
    float4 old[8];
    // all the loads first: their latencies overlap
#pragma unroll
    for (int i = 0; i < 8; ++i)
      old[i] = i < count ? *reinterpret_cast<const float4*>(p + 4 * i * ld)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < count)
        *reinterpret_cast<float4*>(p + 4 * i * ld) =
            make_float4(old[i].x + (v[i].x + b.x), old[i].y + (v[i].y + b.y),
                        old[i].z + (v[i].z + b.z), old[i].w + (v[i].w + b.w));
  }
};

// ---------------------------------------------------------------- causal attention

// The fused QKV projection's epilogue: q and k columns go to qkv [tokens, 3 * width] as bf16
// (the v columns there are left alone); v goes out transposed per head,
// vt[((b * heads + h) * 64 + d) * length + l], keys contiguous, which is the K-major B operand
// of the attention kernel's P.V product. The 32 rows a warp holds are consecutive tokens of one
// sequence (length % 32 == 0), so each store of a v column covers 64 contiguous bytes of vt.
struct LinearQkv {
  static constexpr bool kLines = true;
  const float* bias;
  __nv_bfloat16* out;  // qkv [tokens, 3 * width]: its q and k columns, as whole lines
  __nv_bfloat16* vt;
  int64_t ldo;  // 3 * width
  int64_t width, length, heads;
  // q and k leave as whole 128-byte lines of qkv; the v columns in the row form below
  __device__ __forceinline__ bool is_line(int64_t col) const { return col < 2 * width; }
  __device__ __forceinline__ void pack32(const float (&acc)[32], int64_t col0,
                                         uint32_t (&pk)[16]) const {
    float b[32];
    load_bias32(bias, col0, b);
#pragma unroll
    for (int k = 0; k < 16; ++k)
      pk[k] = pack_bf16x2(acc[2 * k] + b[2 * k], acc[2 * k + 1] + b[2 * k + 1]);
  }
  // v: column d of head h goes to vt row (b * heads + h) * 64 + d at position l; the lanes of
  // a warp hold consecutive tokens, so each store covers 64 contiguous bytes (a lane holds 32
  // consecutive columns of one token's row, inside one head: the head size is 64)
  __device__ __forceinline__ void store_row(const float (&acc)[32], int64_t row, int64_t col0,
                                            int64_t cols) const {
    float b[32];
    load_bias32(bias, col0, b);
    const int64_t hd = col0 - 2 * width;
    const int64_t bi = row / length, l = row - bi * length;
    __nv_bfloat16* dst = vt + ((bi * heads + (hd >> 6)) * 64 + (hd & 63)) * length + l;
#pragma unroll
    for (int j = 0; j < 32; ++j) dst[j * length] = __float2bfloat16_rn(acc[j] + b[j]);
  }
};

// vt[(bh * 64 + d) * length + l] = qkv[(b * length + l) * 3 * width + 2 * width + h * 64 + d]:
// one CTA turns a [64 keys][64 d] block through shared memory (rows padded to 66 elements).
__global__ void __launch_bounds__(256) v_transpose_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                          __nv_bfloat16* __restrict__ vt,
                                                          int64_t length, int64_t heads) {
  __shared__ __nv_bfloat16 tile[64][66];
  const int64_t width = heads * 64;
  const int64_t bh = blockIdx.x, b = bh / heads, h = bh % heads;
  const int64_t l0 = (int64_t)blockIdx.y * 64;
  for (int i = threadIdx.x; i < 64 * 32; i += 256) {
    const int l = i >> 5, d2 = (i & 31) * 2;
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(
        qkv + (b * length + l0 + l) * 3 * width + 2 * width + h * 64 + d2);
    tile[l][d2] = v.x;
    tile[l][d2 + 1] = v.y;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 32; i += 256) {
    const int d = i >> 5, l2 = (i & 31) * 2;
    __nv_bfloat162 v;
    v.x = tile[l2][d];
    v.y = tile[l2 + 1][d];
    *reinterpret_cast<__nv_bfloat162*>(vt + (bh * 64 + d) * length + l0 + l2) = v;
  }
}

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
  const cudaError_t e = ppyb200::launch_pdl(
      embed_kernel, dim3((unsigned)((work + 255) / 256)), dim3(256), 0, stream_now(), ids,
      reinterpret_cast<const __nv_bfloat16*>(wte), reinterpret_cast<const __nv_bfloat16*>(wpe), x,
      tokens, length, width, vocab, status);
  return finish(e, "ppyb200_gpt2_embed", 1);
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
  const bool rows = n % 8 == 0 && aligned16(out) && (bias == nullptr || aligned16(bias));
  const bool lines = rows && n % 64 == 0;
  cudaError_t e;
  if (activation == 1 && lines)
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearBf16Lines<1>{bias, O, n}, status,
                              ppyb200_sm_count(), stream_now());
  else if (lines)
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearBf16Lines<0>{bias, O, n}, status,
                              ppyb200_sm_count(), stream_now());
  else if (activation == 1 && rows)
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearBf16Rows<1>{bias, O, n}, status,
                              ppyb200_sm_count(), stream_now());
  else if (rows)
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearBf16Rows<0>{bias, O, n}, status,
                              ppyb200_sm_count(), stream_now());
  else if (activation == 1)
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
  if (!ppyb200::gemm::tileable(m, n, k) || !aligned16(a) || !aligned16(w)) {
    ppyb200_set_error("ppyb200_linear_residual: K % 64 and 16-byte aligned operands required");
    return PPYB200_RAISED;
  }
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(a);
  const auto* W = reinterpret_cast<const __nv_bfloat16*>(w);
  cudaError_t e;
  if (n % 4 == 0 && aligned16(residual) && (bias == nullptr || aligned16(bias)))
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearResidualQuads{bias, residual, n}, status,
                              ppyb200_sm_count(), stream_now());
  else
    e = ppyb200::gemm::launch(A, W, m, n, k, LinearResidual{bias, residual, n}, status,
                              ppyb200_sm_count(), stream_now());
  return finish(e, "ppyb200_linear_residual", 1);
}

int32_t ppyb200_linear_qkv_bf16(const uint16_t* a, const uint16_t* w, const float* bias,
                                uint16_t* qkv, uint16_t* vt, int64_t m, int64_t k,
                                int64_t length, int64_t heads, int32_t* status) {
  if (m <= 0) return PPYB200_OK;
  const int64_t width = heads * 64, n = 3 * width;
  if (heads <= 0 || length <= 0 || length % 32 != 0 || m % length != 0 ||
      !ppyb200::gemm::tileable(m, n, k) || !aligned16(a) || !aligned16(w) || !aligned16(qkv) ||
      !aligned16(vt) || (bias != nullptr && !aligned16(bias))) {
    ppyb200_set_error("ppyb200_linear_qkv_bf16: K % 64, length % 32, whole sequences and "
                      "16-byte aligned buffers (bias included) required");
    return PPYB200_RAISED;
  }
  LinearQkv epi{bias, reinterpret_cast<__nv_bfloat16*>(qkv), reinterpret_cast<__nv_bfloat16*>(vt),
                3 * width, width, length, heads};
  return finish(ppyb200::gemm::launch(reinterpret_cast<const __nv_bfloat16*>(a),
                                      reinterpret_cast<const __nv_bfloat16*>(w), m, n, k, epi,
                                      status, ppyb200_sm_count(), stream_now()),
                "ppyb200_linear_qkv_bf16", 1);
}

int32_t ppyb200_attention_causal_vt_bf16(const uint16_t* qkv, const uint16_t* vt, uint16_t* out,
                                         int64_t batch, int64_t length, int64_t heads,
                                         int64_t head_dim, int32_t* status) {
  if (batch <= 0 || length <= 0 || heads <= 0) return PPYB200_OK;
  if (!ppyb200::attention::tileable(batch, length, heads, head_dim) || !aligned16(qkv) ||
      !aligned16(vt) || !aligned16(out)) {
    ppyb200_set_error("ppyb200_attention_causal_vt_bf16: head_dim 64, length a multiple of 128 "
                      "and 16-byte aligned buffers required");
    return PPYB200_RAISED;
  }
  return finish(ppyb200::attention::launch(reinterpret_cast<const __nv_bfloat16*>(qkv),
                                           reinterpret_cast<const __nv_bfloat16*>(vt),
                                           reinterpret_cast<__nv_bfloat16*>(out), batch, length,
                                           heads, status, ppyb200_sm_count(), stream_now()),
                "ppyb200_attention_causal_vt_bf16", 1);
}

int32_t ppyb200_attention_causal_bf16(const uint16_t* qkv, uint16_t* out, int64_t batch,
                                      int64_t length, int64_t heads, int64_t head_dim) {
  if (batch <= 0 || length <= 0 || heads <= 0) return PPYB200_OK;
  if (!ppyb200::attention::tileable(batch, length, heads, head_dim) || !aligned16(qkv) ||
      !aligned16(out)) {
    ppyb200_set_error("ppyb200_attention_causal_bf16: head_dim 64, length a multiple of 128 and "
                      "16-byte aligned buffers required");
    return PPYB200_RAISED;
  }
  int32_t* status = ppyb200_status_word();
  void* vt = ppyb200_scratch(batch * heads * 64 * length * 2);
  if (status == nullptr || vt == nullptr) return PPYB200_RAISED;
  const dim3 grid((unsigned)(batch * heads), (unsigned)(length / 64));
  v_transpose_kernel<<<grid, 256, 0, stream_now()>>>(reinterpret_cast<const __nv_bfloat16*>(qkv),
                                                     reinterpret_cast<__nv_bfloat16*>(vt), length,
                                                     heads);
  const int32_t s = finish(cudaGetLastError(), "ppyb200_attention_causal_bf16 (v transpose)", 1);
  if (s != PPYB200_OK) return s;
  return ppyb200_attention_causal_vt_bf16(qkv, reinterpret_cast<const uint16_t*>(vt), out, batch,
                                          length, heads, head_dim, status);
}

}  // extern "C"
