/* ppyb200.h -- the C ABI of the PPy B200 backend.
 *
 * Two kinds of entry points live behind this ABI.
 *
 * 1. libppyb200.so, the runtime every built module uses: device selection, the
 *    launch stream, the per-device scratch arena and status word, cached device
 *    buffers for host-memory calls, and the hand-written kernels that are not
 *    generated per module (the dense matmul, the Collatz-style range reduction).
 *
 * 2. The per-module libraries `ppy build X --backend b200` writes. Each IR function
 *    F of a built module exports
 *
 *        int32_t <symbol>(<atoms of each parameter>..., int64_t *slot);
 *        int32_t <symbol>__device(<atoms of each parameter>..., int64_t *slot);
 *
 *    with the atoms of the reference's native ABI (backend/llvm/from_ir.py:1-13,
 *    the signature tests/test_tensor_fusion.py:269-282 calls through ctypes): a
 *    `buffer<T>` parameter is `T *data, int64_t len`; an `f64`/`f32` scalar is a
 *    `double`/`float`; an `i64` is `int64_t`; a `ptr<T>` is `T *`; the function's
 *    result is written to `*slot`. `<symbol>` takes HOST buffers (it copies what the
 *    function reads to the device, launches, and copies what it writes back);
 *    `<symbol>__device` takes DEVICE buffers and launches on the current stream.
 *    Both return the reference's status (ppy_runtime/abi.py:25-35):
 *    PPYB200_OK, PPYB200_FALLBACK (a guard failed: the caller reruns the function
 *    in CPython, as it does for the LLVM backend), or PPYB200_RAISED (a CUDA error;
 *    ppyb200_last_error() says which).
 *
 * Every function here is thread-safe; the device and stream are per calling thread.
 */
#ifndef PPYB200_H
#define PPYB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PPYB200_ABI_VERSION 1

/* ppy_runtime/abi.py:25-35: STATUS_OK, STATUS_FALLBACK, STATUS_RAISED. */
#define PPYB200_OK 0
#define PPYB200_FALLBACK 1
#define PPYB200_RAISED (-1)

/* ---------------------------------------------------------------- runtime */

/* The ABI version this library implements (PPYB200_ABI_VERSION). */
int32_t ppyb200_abi_version(void);

/* Number of CUDA devices visible, or 0 without a driver or a device. Replaces the
 * device probe of ppy_runtime/cuda.py:146-163 (`available`). */
int32_t ppyb200_device_count(void);

/* Make `device` the calling thread's device (cudaSetDevice) and create its state.
 * Replaces ppy_runtime/cuda.py:51-57 (`Driver` binds device 0's primary context);
 * here every device of the node may be bound, one per calling thread. It also loads the
 * device code and static array of ppyb200_colmax_abs_f32_noalloc onto the device, so that
 * no later call of that entry point allocates. */
int32_t ppyb200_init(int32_t device);

/* The calling thread's device, or -1 before ppyb200_init. */
int32_t ppyb200_current_device(void);

/* The message of the calling thread's last failure ("" when none). Replaces
 * ppy_runtime/cuda.py:36-38 (`CudaError` carries the driver's error string). */
const char *ppyb200_last_error(void);

/* Record a failure message for the calling thread (used by built modules). */
void ppyb200_set_error(const char *message);

/* The stream the calling thread's launches go to: a cudaStream_t, or NULL for the
 * current device's own non-blocking stream. */
int32_t ppyb200_set_stream(void *stream);
void *ppyb200_stream(void);

/* Wait for the calling thread's stream. */
int32_t ppyb200_sync(void);

/* Number of streaming multiprocessors of the current device. */
int32_t ppyb200_sm_count(void);

/* Device memory that a call may use as temporaries, reused by the next call on the
 * same (device, stream): at least `bytes`, 256-byte aligned, NULL on failure. */
void *ppyb200_scratch(int64_t bytes);

/* A zeroed device int32 status word for one call on the current stream (the
 * zeroing is enqueued on that stream). Kernels raise it to PPYB200_FALLBACK. */
int32_t *ppyb200_status_word(void);

/* Read the status word back after the call's kernels (synchronises the stream):
 * PPYB200_OK, PPYB200_FALLBACK, or PPYB200_RAISED when a device function raised (a
 * loop of a parallel body past its trip bound, PPYB200_LOOP_LIMIT trips per index). */
int32_t ppyb200_read_status(int32_t *word);

/* Cached device buffers for host-memory calls. */
void *ppyb200_device_buffer(int64_t bytes);
void ppyb200_release_buffer(void *pointer);

/* Host<->device copies on the current stream (async; ppyb200_sync waits). */
int32_t ppyb200_copy_to_device(void *device_dst, const void *host_src, int64_t bytes);
int32_t ppyb200_copy_to_host(void *host_dst, const void *device_src, int64_t bytes);

/* `rows` rows of `row_bytes` each from device memory (rows `device_pitch` bytes apart) into
 * host memory (rows `host_pitch` bytes apart), one strided copy on the current stream (async):
 * e.g. GPT-2's logits, computed into rows padded to 128-byte lines, into a contiguous host
 * array. The reference's runtime copies whole contiguous arrays (ppy_runtime/cuda.py:125-126, `download`);
 * this is the strided form of that copy-out. */
int32_t ppyb200_copy_rows_to_host(void *host_dst, int64_t host_pitch, const void *device_src,
                                  int64_t device_pitch, int64_t row_bytes, int64_t rows);

/* A second stream of the calling thread's device for pipelining a host-memory call: fork
 * returns it in *side after making it wait for the work already on the current stream; join
 * makes the current stream wait for the work on it. The reference's runtime copies and
 * launches on one synchronous path (ppy_runtime/cuda.py:194-252); built modules use these to
 * overlap one chunk's copies with another's kernel. */
int32_t ppyb200_fork(void **side);
int32_t ppyb200_join(void *side);

/* Translate a cudaError_t into a status, recording `what` when it is a failure. */
int32_t ppyb200_check(int32_t cuda_error, const char *what);

/* Kernels launched through this library and the modules built against it. */
uint64_t ppyb200_launches(void);
void ppyb200_count_launches(uint64_t count);

/* Device allocations (cudaMalloc) this runtime has made since the library loaded: scratch
 * arenas, status words, cached buffers. No counterpart in the reference, whose runtime
 * allocates per launch; it lets a caller check that a call allocated nothing. */
uint64_t ppyb200_device_allocations(void);

/* Programmatic dependent launch: while on (the default), the tensor-core GEMMs, the
 * attention kernel, the GPT-2 embedding and the row-group kernels are launched so that
 * their CTAs may start, and set up, while the kernel before them on the stream drains;
 * each waits (griddepcontrol.wait) for that kernel's results before it touches memory.
 * Results are the same either way. No counterpart in the reference, which launches one
 * kernel per call and waits for it. Process-wide; ppyb200_set_pdl returns the previous
 * setting. */
int32_t ppyb200_set_pdl(int32_t enabled);
int32_t ppyb200_pdl(void);

/* ---------------------------------------------------------------- matmul */

/* C[M,N] = A[M,K] @ B[K,N] (+ bias[N]): bf16 A and B, row-major; f32 bias (NULL for none);
 * f32 accumulation and f32 C. Replaces LowerTensor.op_matmul, the naive i-j-k loop nest
 * of ir/transforms/lower_tensor.py:756-776, for `tensor.matmul` / `linalg.matmul`
 * (ir/dialects/tensor.py:475-488, linalg.py:309-320) of `tensor.convert`ed bf16 operands,
 * with the `tensor.add` of a broadcast bias row FuseTensor leaves after it. Whole
 * 128x256x64 tiles (M % 128, N % 256, K % 64) with a 16-byte aligned A run on tcgen05
 * tensor cores (B is first transposed into the scratch arena); other shapes run on the
 * CUDA cores. Device pointers; enqueued on the current stream. */
int32_t ppyb200_matmul_bf16(const uint16_t *a, const uint16_t *b, const float *bias, float *c,
                            int64_t m, int64_t n, int64_t k);

/* ppyb200_matmul_bf16 with B given K-major, as bt[N,K] (the layout torch.nn.Linear keeps
 * its weight in): tensor cores only; PPYB200_FALLBACK, with nothing launched, for shapes
 * that are not whole tiles or operands not 16-byte aligned. */
int32_t ppyb200_matmul_bf16_kmajor(const uint16_t *a, const uint16_t *bt, const float *bias,
                                   float *c, int64_t m, int64_t n, int64_t k);

/* ppyb200_matmul_bf16_kmajor into rows `ldc` floats apart (ldc >= N): C[i*ldc + j] for
 * j < N, nothing written in the columns N .. ldc-1 of a row. Rows that start on 128-byte
 * lines (C 128-byte aligned, ldc % 32 == 0) store whole lines: GPT-2's logits, 50257 floats a
 * row, go into rows 50272 apart. PPYB200_RAISED for ldc < N. */
int32_t ppyb200_matmul_bf16_kmajor_ld(const uint16_t *a, const uint16_t *bt, const float *bias,
                                      float *c, int64_t ldc, int64_t m, int64_t n, int64_t k);

/* C[M,N] = A[M,K] @ B[K,N] (+ bias[N]) for f32 A, B, bias (NULL for none) and C, row-major:
 * LowerTensor.op_matmul (ir/transforms/lower_tensor.py:756-776) for f32 `tensor.matmul` /
 * `linalg.matmul`, with the bias row FuseTensor leaves after it. On tcgen05 tensor cores as
 * three tf32 products, A_hi B_hi + A_hi B_lo + A_lo B_hi, with x_hi = x rounded to tf32 and
 * x_lo = (x - x_hi) rounded to tf32 (the split operands, 16 (M + N) Kp bytes with Kp = K
 * rounded up to 32, go to the scratch arena): each product term is within about 2^-21 of
 * |a||b| of the f32 product, the sum accumulated in f32. Inputs that are not finite are
 * detected by the split, and C is then recomputed with f32 FMAs in k order (IEEE infinities
 * and NaNs, as the reference's loop). Any M, N, K (K = 0 gives the bias); no alignment
 * needed. Device pointers; enqueued on the current stream (four launches). */
int32_t ppyb200_matmul_f32(const float *a, const float *b, const float *bias, float *c,
                           int64_t m, int64_t n, int64_t k);

/* bt[n*K + k] = b[k*N + n]: a bf16 [K,N] matrix into [N,K] (tiled through shared memory). */
int32_t ppyb200_transpose_bf16(const uint16_t *b, uint16_t *bt, int64_t k, int64_t n);

/* Which tensor-core GEMM kernel every bf16 matmul of this library launches (the matmul entry
 * points, the GPT-2 linear layers, built modules' matmuls): PPYB200_GEMM_BY_SHAPE (the
 * default) clusters of two CTAs per 256 x 256 tile (tcgen05.mma.cta_group::2) when M >= 256
 * and one CTA per 128 x 256 tile otherwise; PPYB200_GEMM_PAIRS and PPYB200_GEMM_SINGLE one of
 * them always. Process-wide; returns the previous form, or PPYB200_RAISED for another value. */
#define PPYB200_GEMM_BY_SHAPE 0
#define PPYB200_GEMM_PAIRS 1
#define PPYB200_GEMM_SINGLE 2
int32_t ppyb200_set_gemm_form(int32_t form);
int32_t ppyb200_gemm_form(void);

/* ---------------------------------------------------------------- GPT-2 pieces */

/* x[t, c] = wte[ids[t], c] + wpe[t % length, c] (bf16 tables, f32 x [tokens, width]): the
 * embedding of examples/46_gpt2/gpt2.ppy:212 (`wte[ids] + wpe[0:length]`). An id outside
 * [0, vocab) reads nothing and raises `*status` (may be NULL) to 2. width % 8 == 0. */
int32_t ppyb200_gpt2_embed(const int64_t *ids, const uint16_t *wte, const uint16_t *wpe,
                           float *x, int64_t tokens, int64_t length, int64_t width,
                           int64_t vocab, int32_t *status);

/* out[M,N] (bf16) = act(a[M,K] @ w[N,K]^T + bias[N]), act 0 = identity, 1 = GELU-tanh, on
 * tcgen05 tensor cores: F.linear (+ F.gelu(approximate="tanh")) of gpt2.ppy:49-56 with the
 * torch.nn.Linear weight layout. K % 64 == 0. `*status` (may be NULL) is raised to 2 if the
 * kernel gives up a bounded wait. */
int32_t ppyb200_linear_bf16(const uint16_t *a, const uint16_t *w, const float *bias,
                            uint16_t *out, int64_t m, int64_t n, int64_t k, int32_t activation,
                            int32_t *status);

/* residual[M,N] (f32) += a[M,K] @ w[N,K]^T + bias[N]: `torch.add(x, F.linear(...))` of
 * gpt2.ppy:54,57, the residual updated in place by the tensor-core epilogue. */
int32_t ppyb200_linear_residual(const uint16_t *a, const uint16_t *w, const float *bias,
                                float *residual, int64_t m, int64_t n, int64_t k,
                                int32_t *status);

/* The fused QKV projection of gpt2.ppy:50-51 (`F.linear(h, w_qkv, b_qkv)` split into q, k, v
 * heads) on tcgen05 tensor cores, written in the layouts ppyb200_attention_causal_vt_bf16
 * reads: q and k as bf16 into qkv [m, 3*heads*64] (its v columns are not written), v as bf16
 * transposed per head into vt [batch*heads*64, length]: vt[((b*heads + h)*64 + d)*length + l]
 * = v of token b*length + l, head h, dimension d. m = batch*length whole sequences,
 * length % 32 == 0, K % 64 == 0, w [3*heads*64, K]. */
int32_t ppyb200_linear_qkv_bf16(const uint16_t *a, const uint16_t *w, const float *bias,
                                uint16_t *qkv, uint16_t *vt, int64_t m, int64_t k,
                                int64_t length, int64_t heads, int32_t *status);

/* Causal self-attention, F.scaled_dot_product_attention(q, k, v, is_causal=True) of
 * gpt2.ppy:52, on tcgen05 tensor cores (S = Q K^T and O += P V in tensor memory, f32 online
 * softmax): q, k from qkv [batch*length, 3*heads*64] (head h at columns h*64 of each), v from
 * vt as ppyb200_linear_qkv_bf16 writes it; out [batch*length, heads*64] bf16 (heads merged,
 * as gpt2.ppy:53). head_dim 64, length % 128 == 0. `*status` (may be NULL) is raised to 2 if
 * the kernel gives up a bounded wait. */
int32_t ppyb200_attention_causal_vt_bf16(const uint16_t *qkv, const uint16_t *vt, uint16_t *out,
                                         int64_t batch, int64_t length, int64_t heads,
                                         int64_t head_dim, int32_t *status);

/* The same attention from qkv alone (q, k, v side by side): v is first transposed into the
 * scratch arena; a bounded wait given up raises the call's status word
 * (ppyb200_status_word). */
int32_t ppyb200_attention_causal_bf16(const uint16_t *qkv, uint16_t *out, int64_t batch,
                                      int64_t length, int64_t heads, int64_t head_dim);

/* ---------------------------------------------------------------- tensor parallel over NVLink */

/* Bytes of the handle ppyb200_shared_alloc writes (a cudaIpcMemHandle_t). */
#define PPYB200_SHARED_HANDLE_BYTES 64

/* Zeroed device memory other processes on this node can map: its handle is written into
 * handle[PPYB200_SHARED_HANDLE_BYTES]; NULL on failure (message in ppyb200_last_error). */
void *ppyb200_shared_alloc(int64_t bytes, uint8_t *handle);
void ppyb200_shared_free(void *pointer);
/* Another process's ppyb200_shared_alloc memory mapped into the current device (peer access
 * over NVLink); NULL on failure. */
void *ppyb200_shared_open(const uint8_t *handle);
void ppyb200_shared_close(void *pointer);

/* The row-parallel linear of GPT-2's tensor-parallel variant (the out and proj projections of
 * gpt2.ppy:54,57 with their input columns split over `ranks`), one fused kernel: this rank's
 * partial product a[M,K] @ w[N,K]^T (bf16 in, f32) on tcgen05 tensor cores, every 16-byte
 * piece of it stored by the epilogue into slots[s] for s < ranks -- slots[s] is this rank's
 * slot in rank s's exchange buffer, local or a peer's mapped by ppyb200_shared_open, each
 * [M, N] f32. K % 64 == 0, N % 4 == 0, ranks <= 8; `slots` is a host array. `*status` (may
 * be NULL) is raised to 2 if the kernel gives up a bounded wait. */
int32_t ppyb200_tp_partial_scatter(const uint16_t *a, const uint16_t *w, float *const *slots,
                                   int32_t ranks, int64_t m, int64_t n, int64_t k,
                                   int32_t *status);

/* After the stream's earlier work: `epoch` into element `rank` of flags[s] (every rank's
 * int32 flag array, mapped here) for s < ranks, with system-scope release. */
int32_t ppyb200_tp_signal(int32_t *const *flags, int32_t ranks, int32_t rank, int32_t epoch);

/* Waits (bounded, about 2 s) until flags[0..ranks) of this rank's flag array reach `epoch`,
 * then x[M,N] += bias[N] + exchange[0] + exchange[1] + ... (slot s at s*M*N floats), summed
 * in rank order on every rank. A wait given up raises `*status` (may be NULL) to 2 and leaves
 * x alone. N % 4 == 0; x, bias (may be NULL) and exchange 16-byte aligned. */
int32_t ppyb200_tp_accumulate(float *x, const float *bias, const float *exchange,
                              const int32_t *flags, int32_t ranks, int64_t m, int64_t n,
                              int32_t epoch, int32_t *status);

/* The reduce-scatter form of the same exchange, (R - 1) / R of the partial sent twice instead
 * of all of it R - 1 times (R = ranks). Rows split into blocks of ceil(M / R); block s belongs to
 * rank s.
 *
 * ppyb200_tp_partial_reduce_scatter: as ppyb200_tp_partial_scatter, but the epilogue stores
 * the rows of block s only, into slots[s] -- this rank's slot in rank s's exchange buffer,
 * [ceil(M / R), N] f32.
 * Then ppyb200_tp_signal on the first flag set.
 *
 * ppyb200_tp_reduce_block: waits (bounded) until flags[0..ranks) reach `epoch`, then for the
 * rows of block `rank`: x += bias + exchange[0] + exchange[1] + ... (slot s at
 * s * ceil(M / R) * N floats, rank order: the sum ppyb200_tp_accumulate makes), and the result
 * into gather[s] for every s != rank (this rank's slot in rank s's gather buffer, same shape).
 * Then ppyb200_tp_signal on the second flag set.
 *
 * ppyb200_tp_gather_blocks: waits (bounded) until flags[0..ranks) reach `epoch`, then copies
 * slot s of `gathered` (this rank's gather buffer, written by rank s) into block s of x for
 * every s != rank. `gather`/`slots` are host arrays; a wait given up raises `*status` (may be
 * NULL) to 2 and leaves x alone. N % 4 == 0, pointers 16-byte aligned. */
int32_t ppyb200_tp_partial_reduce_scatter(const uint16_t *a, const uint16_t *w,
                                          float *const *slots, int32_t ranks, int64_t m,
                                          int64_t n, int64_t k, int32_t *status);
int32_t ppyb200_tp_reduce_block(float *x, const float *bias, const float *exchange,
                                float *const *gather, const int32_t *flags, int32_t ranks,
                                int32_t rank, int64_t m, int64_t n, int32_t epoch,
                                int32_t *status);
int32_t ppyb200_tp_gather_blocks(float *x, const float *gathered, const int32_t *flags,
                                 int32_t ranks, int32_t rank, int64_t m, int64_t n,
                                 int32_t epoch, int32_t *status);

/* ---------------------------------------------------------------- measurement */

/* The issue ceiling of the Collatz step body of the parallel.range reduction (the reference's
 * collatz_sum__par1 in tests/golden/collatz.ppyir: the x != 1 and parity tests, x / 2 or the
 * checked 3x + 1, the checked step count, the trip bound): every lane of a full grid runs four
 * independent chains of that step, branch-free, `steps_per_chain` steps each, so nothing
 * diverges. `checksum` is a device int64 the kernel may add to (keeps the chains live);
 * *total_steps (host) receives the steps the launch performs. No counterpart in the reference:
 * the benchmark divides the reduction's steps/s by this kernel's to give its roofline fraction.
 * Enqueued on the current stream. */
int32_t ppyb200_collatz_step_peak(int64_t steps_per_chain, int64_t *checksum,
                                  int64_t *total_steps);

/* ---------------------------------------------------------------- without allocation */

/* Floats in the fixed device array ppyb200_colmax_abs_f32_noalloc keeps its partials in. */
#define PPYB200_NOALLOC_PARTIALS 262144

/* out[c] = max over r of |x[r*cols + c]| (NaN-propagating, -inf for no rows): the
 * leading-axis reduction the backend builds for tensor.reduce(abs(x), axes=(0,), op="max"),
 * for callers that cannot allocate device memory at call time (memory reserved once at
 * start-up, or owned by another framework's allocator). It has no counterpart in the
 * reference: it exists for those callers. It allocates nothing -- its partial results live
 * in a static 1 MiB __device__ array (PPYB200_NOALLOC_PARTIALS floats) that every GPU
 * loading this library holds until exit -- and refuses rows wider than
 * PPYB200_NOALLOC_PARTIALS columns with PPYB200_RAISED. CUDA loads device code lazily, and
 * loading this entry point's module (the array with it) takes device memory: ppyb200_init
 * does that for the device it binds, and looks up the array's address there
 * (cudaGetSymbolAddress), so that after ppyb200_init no call allocates, through this
 * library or the driver. Without ppyb200_init the first call on each device does the
 * set-up: make that call before the caller reserves its memory and before any stream
 * capture. All calls share the array; calls that overlap on the GPU race on it. Device
 * pointers; enqueued on the current stream. */
int32_t ppyb200_colmax_abs_f32_noalloc(const float *x, int64_t rows, int64_t cols, float *out);

#ifdef __cplusplus
}
#endif

#endif /* PPYB200_H */
