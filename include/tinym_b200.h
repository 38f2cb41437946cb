/*
 * tinym_b200.h -- C ABI of the B200 (sm_100a) tiny-M FP8 GEMM.
 *
 *     Y[M,N] = bf16( alpha * sum_k X[m,k] * W[n,k] )
 *
 * X is [M,K] and W is [N,K], both row-major float8 E4M3 (OCP "e4m3fn"
 * encoding: no infinities, 0x7F/0xFF are NaN).  Accumulation is FP32 and Y
 * is row-major BF16 with row stride ldy (>= N) elements.  alpha is the
 * per-tensor scale product x_scale * w_scale.
 *
 * This library replaces the reference's native boundary:
 *   - the torch op body fp8_gemm_cuda / check_inputs / 6-shape dispatch
 *     (src/torch_candidate_extension.cu:17-81), and
 *   - the templated launchers FP8GemmTinyM<...>::run and
 *     FP8GemmTinyMMmaM16<...>::run with their C-style wrapper
 *     sm120_tinym_mma_m16_run (include/fp8_gemm_tinym.cuh:724-824).
 * Unlike those, shapes are runtime values: 1 <= M <= 16, any N >= 1, any
 * K >= 16 with K % 16 == 0 (TMA row-stride rule).  The dispatch table
 * (tinym_select_plan) picks the kernel and its tiling per shape.
 *
 * Conventions (every entry point):
 *   - Returns a tinym_status code (0 = TINYM_OK).  No C++ exception ever
 *     crosses this boundary.  On failure, tinym_last_error() returns a
 *     message for the calling thread.
 *   - Launches are asynchronous on the given cudaStream_t (passed as
 *     void*; NULL = legacy default stream) on the calling thread's current
 *     CUDA device.  Pointers are device pointers on that device.
 *   - X and W must be 16-byte aligned; Y must be 2-byte aligned.
 *   - Inputs are borrowed; nothing is retained after the call returns
 *     except cached TMA descriptors keyed by (pointer, shape).
 *   - The library allocates no device memory on the call path.  The first
 *     GEMM call on a device allocates one pinned, device-mapped 4-byte host
 *     word (the pending-error word, see tinym_pending_errors); the
 *     no-allocation entry point never does.
 */
#ifndef TINYM_B200_H
#define TINYM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TINYM_ABI_VERSION 8

/* Exported-symbol marker (the library is built with hidden visibility). */
#if defined(__GNUC__)
#define TINYM_API __attribute__((visibility("default")))
#else
#define TINYM_API
#endif

typedef enum tinym_status {
    TINYM_OK = 0,
    TINYM_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, bad ldy */
    TINYM_ERR_UNSUPPORTED_SHAPE = 2, /* M outside 1..16 or K % 16 != 0 */
    TINYM_ERR_MISALIGNED = 3,        /* X/W not 16-byte or Y not 2-byte aligned */
    TINYM_ERR_CUDA = 4,              /* a CUDA runtime/driver call failed */
    TINYM_ERR_UNSUPPORTED_DEVICE = 5,/* current device is not sm_100 */
    TINYM_ERR_DEVICE_TIMEOUT = 6,    /* a bounded device-side wait expired */
    TINYM_ERR_BAD_PLAN = 7           /* an explicit plan is inconsistent */
} tinym_status;

/* Kernel families (tinym_plan.kernel). */
#define TINYM_KERNEL_TC 1      /* tcgen05 swap-AB: W tile = MMA A (M=128), X = MMA B */
#define TINYM_KERNEL_SIMT_M1 2 /* M == 1 only: CUDA-core dequantise + FP32 FMA */

/* A launch plan: which kernel and how the problem is cut.  Produced by
 * tinym_select_plan (the shape-dispatch table, replacing the hard-coded
 * six-way template dispatch of src/torch_candidate_extension.cu:60-78) and
 * accepted back by tinym_fp8_gemm_ex for sweeps. */
typedef struct tinym_plan {
    int32_t kernel;         /* TINYM_KERNEL_* */
    int32_t split_k;        /* CTAs per W tile (K split, 1..8); >1 => cluster of split_k CTAs */
    int32_t stages;         /* shared-memory ring depth (W+X stages) */
    int32_t mma_n;          /* TC: MMA N (8 or 16, >= M); SIMT: 0 */
    int32_t consumer_warps; /* SIMT: dequant/FMA warps (4 or 8); TC: 0 */
    int32_t block_k;        /* K bytes per stage: 128, or 256 / 512 (TC, K % 128 == 0); 0 = 128 */
    int32_t tile_m;         /* W rows per CTA tile (= MMA M): 128, or 64 (TC); 0 = 128 */
    int32_t tiles_n;        /* out: ceil(N / tile_m) */
    int32_t grid_ctas;      /* out: CTAs launched = tiles_n * split_k */
    int32_t smem_bytes;     /* out: dynamic shared memory per CTA */
    int32_t threads;        /* out: threads per CTA */
} tinym_plan;

/* Y = (x_scale * w_scale) * X . W^T.  Mirrors FP8GemmTinyM::run /
 * FP8GemmTinyMMmaM16::run (include/fp8_gemm_tinym.cuh:514-518,314-318):
 * same operands, same scale pair, same stream argument. */
TINYM_API int tinym_fp8_gemm(const void* x, const void* w, void* y,
                   int64_t m, int64_t n, int64_t k,
                   float x_scale, float w_scale, void* stream);

/* As tinym_fp8_gemm, but alpha is read on the device from alpha_dev (one
 * FP32 value) when the kernel runs, so no host synchronisation is needed to
 * obtain it.  Replaces the torch op run(Tensor a, Tensor b, float alpha)
 * plus the adapter's alpha.item() cache (candidate_kernel.py:77-102). */
TINYM_API int tinym_fp8_gemm_dev_alpha(const void* x, const void* w, void* y,
                             int64_t m, int64_t n, int64_t k,
                             const float* alpha_dev, void* stream);

/* Full form: explicit output row stride, alpha either on the device
 * (alpha_dev != NULL) or by value, and an optional plan (NULL = use the
 * dispatch table).  Used by the N-sharded wrapper (writes its column slab
 * of a wider Y) and by tuning sweeps.  No reference counterpart beyond the
 * launchers above. */
TINYM_API int tinym_fp8_gemm_ex(const void* x, const void* w, void* y, int64_t ldy,
                      int64_t m, int64_t n, int64_t k,
                      const float* alpha_dev, float alpha,
                      const tinym_plan* plan, void* stream);

/* tinym_fp8_gemm_ex with behaviour flags (TINYM_FLAG_*).
 *
 * TINYM_FLAG_STATIC_W: the caller guarantees that the kernel queued just
 * before this GEMM on the stream does not write W (the usual case for
 * inference weights).  The GEMM then starts streaming W as soon as its CTAs
 * are resident -- under programmatic dependent launch that is during the
 * previous kernel's tail -- and waits for the previous kernel only before
 * it reads X and alpha and writes Y.  Without the flag nothing is read
 * before the previous kernel has completed.  When plan is NULL the dispatch
 * then also packs two CTAs per SM (a 64 KiB ring each, twice the K split),
 * so consecutive GEMMs overlap. */
#define TINYM_FLAG_STATIC_W 1u

/* The plan tinym_fp8_gemm_ex2 would use with these flags (host-only). */
TINYM_API int tinym_select_plan_ex(int64_t m, int64_t n, int64_t k, int32_t sm_count,
                                   uint32_t flags, tinym_plan* out);
TINYM_API int tinym_fp8_gemm_ex2(const void* x, const void* w, void* y, int64_t ldy,
                                 int64_t m, int64_t n, int64_t k,
                                 const float* alpha_dev, float alpha,
                                 const tinym_plan* plan, uint32_t flags, void* stream);

/* The shape-dispatch table: fills *out with the plan tinym_fp8_gemm would
 * use for (m, n, k) on a GPU with sm_count SMs.  Host-only logic (needs no
 * GPU).  Replaces src/torch_candidate_extension.cu:40-46,60-78. */
TINYM_API int tinym_select_plan(int64_t m, int64_t n, int64_t k, int32_t sm_count,
                      tinym_plan* out);

/* Validate a plan for (m, n, k) and fill its derived fields.  Host-only. */
TINYM_API int tinym_check_plan(int64_t m, int64_t n, int64_t k, tinym_plan* plan);

/* How many clusters of `plan` (for this M, N, K) the current device can
 * hold resident at once (CTAs for split_k == 1), from the CUDA occupancy
 * calculator.  A grid of tiles_n clusters runs in one wave when this is
 * >= tiles_n; the automatic dispatch shrinks split_k until it is.  No
 * reference counterpart (the reference launches at most one CTA per SM,
 * include/fp8_gemm_tinym.cuh:757-766). */
TINYM_API int tinym_plan_max_active_clusters(int64_t m, int64_t n, int64_t k,
                                             const tinym_plan* plan, int32_t* out);

/* The plan a call with no explicit plan runs on the current device, with
 * these flags (0 or TINYM_FLAG_STATIC_W): the dispatch table's plan, then
 * split_k lowered (as the launcher does) until every cluster of the grid
 * is resident at once, to the next split that still gives every CTA some
 * K.  Equal to tinym_select_plan_ex(..., device SM count, ...) whenever the
 * device holds that plan's clusters.  Queries the device (occupancy
 * calculator); launches nothing.  No reference counterpart (the reference
 * picks one of six compile-time configurations,
 * src/torch_candidate_extension.cu:60-78). */
TINYM_API int tinym_launch_plan(int64_t m, int64_t n, int64_t k, uint32_t flags,
                                tinym_plan* out);

/* Device error word of the current device: bit flags set by kernels whose
 * bounded waits expired (0 = none).  Synchronises the device.  clear != 0
 * resets the word.  The reference has no counterpart (its waits spin
 * forever, include/fp8_gemm_tinym.cuh:164-176). */
TINYM_API int tinym_device_status(uint32_t* flags, int32_t clear);

/* Pending errors of the current device, without synchronising: the bits of
 * bounded waits that ran out in kernels that have already finished (0 =
 * none), read from a pinned host word that those kernels write at system
 * scope.  Returns TINYM_ERR_DEVICE_TIMEOUT when any bit is set; clear != 0
 * resets the word.  A caller checks it before each launch so that the
 * unspecified output of a timed-out GEMM is reported at the next call (the
 * torch ops raise RuntimeError) instead of being used silently.  Reflects
 * only kernels launched after the device's first GEMM call (which creates
 * the word); tinym_device_status sees every kernel.  No reference
 * counterpart (the reference's waits spin forever). */
TINYM_API int tinym_pending_errors(uint32_t* flags, int32_t clear);

/* Failure-detection self-test: launches the GEMM (plan = NULL for the
 * dispatch table's choice) with fault injection that makes the producer
 * issue no copies, so every consumer wait runs out after timeout_ns
 * (1 .. 1e10 ns).  The kernel then sets bits in the device error word,
 * releases its tensor memory and exits; no GPU fault occurs and the context
 * stays usable.  Read the bits with tinym_device_status.  Y is left
 * unspecified.  No reference counterpart (the reference's waits are
 * unbounded). */
TINYM_API int tinym_selftest_wait_timeout(const void* x, const void* w, void* y,
                                          int64_t m, int64_t n, int64_t k,
                                          const tinym_plan* plan, uint64_t timeout_ns,
                                          void* stream);

/* Packed weight layout.  W is cut into 128-row tiles and 128-byte K chunks;
 * chunk c of tile t is one contiguous [128 rows][128 B] block at byte offset
 * (t * KC + c) * 16384, KC = ceil(K / 128) rounded up to a multiple of 4,
 * zero-filled past N and K.  Each pipeline stage of the TC kernel is then
 * one contiguous HBM range.  The
 * reference's prepare_weights hook (candidate_kernel.py:68-74, a validated
 * identity there; harness fp8_gemm_task_harness.py:13-19 runs it once,
 * untimed) is where a caller repacks.  No reference counterpart beyond
 * that hook. */

/* Size in bytes of the packed form of an [N, K] weight. */
TINYM_API int tinym_packed_weight_bytes(int64_t n, int64_t k, int64_t* bytes);

/* Repack row-major W [N, K] into w_packed (tinym_packed_weight_bytes bytes,
 * 16-byte aligned), asynchronously on `stream`. */
TINYM_API int tinym_pack_weights(const void* w, void* w_packed, int64_t n, int64_t k,
                                 void* stream);

/* tinym_fp8_gemm_ex with W in the packed layout (TC plans only). */
TINYM_API int tinym_fp8_gemm_packed(const void* x, const void* w_packed, void* y, int64_t ldy,
                                    int64_t m, int64_t n, int64_t k,
                                    const float* alpha_dev, float alpha,
                                    const tinym_plan* plan, void* stream);

/* Fused activation path (quantise + GEMM).  The caller's step before the
 * GEMM -- per-tensor E4M3 quantisation of the activation, the harness's
 * quantize_per_tensor (fp8_gemm_task_harness.py:41-44) -- runs as a
 * one-cluster prologue kernel that releases the GEMM at once; the GEMM
 * streams W while X is quantised and waits only before loading X.  The
 * workspace (tinym_quant_workspace_bytes, 256-byte aligned) receives
 * x_scale (f32 at byte 0), alpha = x_scale * w_scale (f32 at byte 4) and
 * the E4M3 codes of X ([M, K] at byte 256).  No reference counterpart: the
 * reference takes pre-quantised X. */
#define TINYM_ACT_BF16 1 /* X is [M, K] bfloat16 */
#define TINYM_ACT_F32 2  /* X is [M, K] float32 */

/* Workspace bytes of tinym_fp8_gemm_quant_act for an [M, K] activation. */
TINYM_API int tinym_quant_workspace_bytes(int64_t m, int64_t k, int64_t* bytes);

/* Y = bf16(alpha * q(X) . W^T) with q(X), x_scale and alpha computed on the
 * device from the BF16 / FP32 activation x_act (16-byte aligned) and the
 * device scalar w_scale_dev.  W is row-major [N, K] E4M3; plan as in
 * tinym_fp8_gemm_ex (NULL = dispatch table). */
TINYM_API int tinym_fp8_gemm_quant_act(const void* x_act, int32_t act_dtype, const void* w,
                                       const float* w_scale_dev, void* y, int64_t ldy,
                                       int64_t m, int64_t n, int64_t k, void* workspace,
                                       const tinym_plan* plan, void* stream);

/* tinym_fp8_gemm_quant_act without a caller-provided workspace, for callers
 * that cannot allocate device memory (an allocator-less runtime, a caller
 * inside a memory pool it does not own).  No counterpart in the reference.
 * The workspace is a static device array inside the library (its address
 * found per device with cudaGetSymbolAddress on the device's first such
 * call, which should therefore come before any stream capture), so the call
 * allocates nothing and needs no workspace argument.  M * K must be at most
 * 524288 (else TINYM_ERR_UNSUPPORTED_SHAPE).  The array is shared by every
 * call on a device and keeps the last call's contents: calls must be
 * ordered on one stream (or otherwise serialised), since calls that overlap
 * on the GPU race.  x_scale and alpha are not observable in this form.  The
 * cached address assumes the device's primary context and no
 * cudaDeviceReset while the library is loaded. */
TINYM_API int tinym_fp8_gemm_quant_act_noalloc(const void* x_act, int32_t act_dtype,
                                               const void* w, const float* w_scale_dev,
                                               void* y, int64_t ldy, int64_t m, int64_t n,
                                               int64_t k, const tinym_plan* plan, void* stream);

/* Fused all-gather of the N-sharded (column-parallel) wrapper.  Rank r owns
 * W rows [col0, col0 + n_local) and, instead of writing a local slab that a
 * collective then gathers, its GEMM epilogue stores the BF16 rows straight
 * into every rank's full Y [M, n_full] (plain stores through CUDA IPC
 * mappings over NVLink) and then adds the number of elements it stored to
 * every rank's 64-bit arrival counter (release, system scope).  One CTA of
 * the GEMM waits (acquire, bounded: 1 s, then bit 0x40 of the device error
 * word) until this rank's counter reaches `target`, so the GEMM completes
 * only when this rank's full Y is present; the grid must fit the GPU in one
 * wave (else TINYM_ERR_BAD_PLAN).
 * Counters only grow: every call adds M * n_full to every rank's counter,
 * so target = the sum of M * n_full over this and all earlier calls (the
 * same on every rank, which make the same calls in the same order).  Two Y
 * buffers used alternately (by e's parity) keep a fast rank's next call
 * from overwriting a result another rank is still reading, provided each
 * rank's readers of Y are stream-ordered before its next call.  No
 * reference counterpart: the reference is single-GPU. */
typedef struct tinym_gather_desc {
    int32_t world;      /* ranks, 1..8 */
    int32_t rank;       /* this rank */
    int64_t n_full;     /* columns (and row stride) of the full Y */
    int64_t col0;       /* first column of this rank's slab */
    void* y_full[8];    /* every rank's full Y for this call, mapped into this process */
    void* flag[8];      /* every rank's 8-byte arrival counter, mapped into this process */
    uint64_t target;    /* this rank's counter once the gather of this call is complete */
} tinym_gather_desc;

/* Y_full (on every rank) = alpha * X . W^T, W N-sharded across the ranks. */
TINYM_API int tinym_fp8_gemm_allgather(const void* x, const void* w_local, int64_t m,
                                       int64_t n_local, int64_t k, const float* alpha_dev,
                                       float alpha, const tinym_gather_desc* gd,
                                       const tinym_plan* plan, void* stream);

/* CUDA IPC helpers for the descriptor: the handle (64 bytes) of the
 * allocation that holds ptr and ptr's offset in it; open / close a peer's
 * handle in this process. */
TINYM_API int tinym_ipc_export(const void* ptr, void* handle, int64_t* offset);
TINYM_API int tinym_ipc_open(const void* handle, void** base);
TINYM_API int tinym_ipc_close(void* base);

/* Human-readable name of a tinym_status code (static string). */
TINYM_API const char* tinym_status_string(int32_t status);

/* Message for the last failing call on this thread ("" if none). */
TINYM_API const char* tinym_last_error(void);

/* TINYM_ABI_VERSION of the loaded library. */
TINYM_API int32_t tinym_abi_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* TINYM_B200_H */
