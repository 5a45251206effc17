/* ORACLE -- test infrastructure only. Nothing in the product (ppy_b200/) links, loads
 * or calls this file; it is the checker the parity tests and bench.py's CPU-baseline
 * leg compare against.
 *
 * A plain-C restatement of what PPy's reference CPU path computes for the hot path,
 * written from the reference's lowering rules:
 *
 *   - tensor.fused maps: one loop over the elements, the body's scalar operations in
 *     IR order, one rounding per f32 operation (ir/transforms/lower_tensor.py:527-608;
 *     backend/llvm/from_ir.py emits plain fadd/fmul/fdiv and llvm.exp.f32 -> expf).
 *   - tensor.reduce / fused reduce: the identity, then every element folded in
 *     row-major order (lower_tensor.py:733-754, :1841-1870); max/min NaN-propagating
 *     (ir/dialects/tensor.py:684-701).
 *   - tensor.matmul: C[i,j] = 0, then += A[i,k]*B[k,j] for k in order
 *     (lower_tensor.py:756-776).
 *   - parallel.reduce of a Collatz body: steps per start with int64 arithmetic checked
 *     for overflow (overflow="python" takes the fallback, from_ir.py:757-771); chunks
 *     fold with wrapping add (ir/transforms/lower_parallel.py:202-208).
 *
 * The *_omp variants split the outer loop across OpenMP threads the way the reference's
 * `parallel` worker pool chunks contiguous ranges (backend/llvm/parallel.py:72-83); they
 * are the CPU baseline, and give the same answer as the serial loops (row-parallel
 * work does not change any fold order).
 *
 * Build: oracle/Makefile (gcc -O2 -fno-fast-math -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define STATUS_OK 0
#define STATUS_FALLBACK 1

static inline float ext_max_f(float a, float c) {
  float chosen = (a >= c) ? a : c;
  return (a == a) ? chosen : a;
}

/* ---------------------------------------------------------------- GELU chain
 * The body of tests/golden/gelu.ppyir: z = a*b + c;
 * y = (0.5*z) * (1 + (1 - 2/(exp(2*(k*(z + 0.044715*(z*(z*z))))) + 1))). */
static inline float gelu_body(float a, float b, float c) {
  const float k0 = (float)0.7978845608028654, k1 = (float)0.044715, two = 2.0f, one = 1.0f,
              half = 0.5f;
  float z = a * b;
  z = z + c;
  float z2 = z * z;
  float z3 = z * z2;
  float t = k1 * z3;
  t = z + t;
  t = k0 * t;
  t = two * t;
  float e = expf(t);
  e = e + one;
  float q = two / e;
  float th = one - q;
  float h = half * z;
  float s = one + th;
  return h * s;
}

void oracle_gelu_chain(const float* a, const float* b, const float* c, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = gelu_body(a[i], b[i], c[i]);
}

void oracle_gelu_chain_omp(const float* a, const float* b, const float* c, float* out, int64_t n,
                           int threads) {
#pragma omp parallel for schedule(static) num_threads(threads)
  for (int64_t i = 0; i < n; ++i) out[i] = gelu_body(a[i], b[i], c[i]);
}

/* ---------------------------------------------------------------- softmax -> layernorm
 * The IR of tests/golden/rows.ppyir, one row at a time, every reduction a row-major
 * fold from its identity, every elementwise group in its body's order:
 *   m = max_j x;  e = exp(x - m);  s = sum_j e;  p = e / s;
 *   mean = (sum_j p) / C;  d = p - mean;  var = (sum_j d*d) / C;
 *   y = ((d * (1 / sqrt(var + eps))) * gamma) + beta                                */
static void softmax_layernorm_row(const float* x, const float* gamma, const float* beta,
                                  float* out, int64_t cols, float* e, float* p) {
  const float C = (float)cols, eps = (float)1e-05, one = 1.0f;
  float m = -INFINITY;
  for (int64_t j = 0; j < cols; ++j) m = ext_max_f(m, x[j]);
  for (int64_t j = 0; j < cols; ++j) e[j] = expf(x[j] - m);
  float s = 0.0f;
  for (int64_t j = 0; j < cols; ++j) s = s + e[j];
  for (int64_t j = 0; j < cols; ++j) p[j] = e[j] / s;
  float t = 0.0f;
  for (int64_t j = 0; j < cols; ++j) t = t + p[j];
  /* fused: d = p - t / C (the body recomputes t / C per element) */
  for (int64_t j = 0; j < cols; ++j) e[j] = p[j] - t / C; /* e now holds d */
  float v = 0.0f;
  for (int64_t j = 0; j < cols; ++j) v = v + e[j] * e[j];
  for (int64_t j = 0; j < cols; ++j) {
    float var = v / C;
    float r = var + eps;
    r = sqrtf(r);
    r = one / r;
    float y = e[j] * r;
    y = y * gamma[j];
    out[j] = y + beta[j];
  }
}

void oracle_softmax_layernorm(const float* x, const float* gamma, const float* beta, float* out,
                              int64_t rows, int64_t cols, float* work) {
  for (int64_t r = 0; r < rows; ++r)
    softmax_layernorm_row(x + r * cols, gamma, beta, out + r * cols, cols, work, work + cols);
}

void oracle_softmax_layernorm_omp(const float* x, const float* gamma, const float* beta,
                                  float* out, int64_t rows, int64_t cols, float* work,
                                  int threads) {
#pragma omp parallel num_threads(threads)
  {
    int me = 0;
#ifdef _OPENMP
    me = omp_get_thread_num();
#endif
    float* mine = work + (int64_t)me * 2 * cols;
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
      softmax_layernorm_row(x + r * cols, gamma, beta, out + r * cols, cols, mine, mine + cols);
  }
}

/* ---------------------------------------------------------------- matmul + bias
 * tensor.matmul then tensor.add of a [N] bias broadcast over rows (matmul.ppyir). */
void oracle_matmul_bias(const float* a, const float* b, const float* bias, float* c, int64_t m,
                        int64_t n, int64_t k) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) c[i * n + j] = 0.0f;
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j)
      for (int64_t q = 0; q < k; ++q) c[i * n + j] = c[i * n + j] + a[i * k + q] * b[q * n + j];
  if (bias != 0)
    for (int64_t i = 0; i < m; ++i)
      for (int64_t j = 0; j < n; ++j) c[i * n + j] = c[i * n + j] + bias[j];
}

/* ---------------------------------------------------------------- Collatz
 * The outlined body of collatz_sum in tests/golden/collatz.ppyir for one start:
 * while x != 1: x = x//2 if x%2 == 0 else 3*x + 1 (mul, add checked); steps += 1
 * (checked). Returns STATUS_FALLBACK on int64 overflow. */
static inline int collatz_steps(int64_t start, int64_t* steps_out) {
  int64_t x = start, steps = 0;
  while (x != 1) {
    if ((x & 1) == 0) {
      x = x >> 1; /* floor division by 2 */
    } else {
      int64_t t;
      if (__builtin_mul_overflow((int64_t)3, x, &t)) return STATUS_FALLBACK;
      if (__builtin_add_overflow(t, (int64_t)1, &x)) return STATUS_FALLBACK;
    }
    if (__builtin_add_overflow(steps, (int64_t)1, &steps)) return STATUS_FALLBACK;
  }
  *steps_out = steps;
  return STATUS_OK;
}

/* Sum and max of the step counts over [lo, hi). Start values <= 0 never reach 1 in the
 * reference either; callers pass lo >= 1. */
int oracle_collatz(int64_t lo, int64_t hi, int64_t* sum_out, int64_t* max_out, int threads) {
  int64_t total = 0, best = 0;
  int failed = 0;
#pragma omp parallel for schedule(dynamic, 4096) reduction(+ : total) reduction(max : best) \
    reduction(| : failed) num_threads(threads)
  for (int64_t s = lo; s < hi; ++s) {
    int64_t steps = 0;
    if (collatz_steps(s, &steps) != STATUS_OK) {
      failed = 1;
      continue;
    }
    total = (int64_t)((uint64_t)total + (uint64_t)steps);
    if (steps > best) best = steps;
  }
  *sum_out = total;
  *max_out = best;
  return failed ? STATUS_FALLBACK : STATUS_OK;
}

/* Step count per start, for the parallel.for form (collatz_steps in collatz.ppyir). */
int oracle_collatz_steps(int64_t lo, int64_t hi, int64_t* out) {
  for (int64_t s = lo; s < hi; ++s)
    if (collatz_steps(s, &out[s - lo]) != STATUS_OK) return STATUS_FALLBACK;
  return STATUS_OK;
}
