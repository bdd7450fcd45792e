/*
 * kebab-b200 C ABI — the drop-in boundary of the B200 GEMM ladder.
 *
 * Plain C: pointers, sizes and an opaque stream handle (binary-compatible
 * with cudaStream_t). All matrix pointers are DEVICE pointers owned by the
 * caller; A and B are read-only, C is written in full (no alpha/beta). Calls
 * are asynchronous on `stream` (NULL = legacy default stream) and return a
 * status code; the message of the last failure on the calling thread is
 * available from kebab_last_error().
 *
 * Layout conventions follow the reference operator (kebab/include/kebab/cuda/
 * cuda_gemm.h:10-33, kebab/lib/cuda/cuda_gemm.cu:112-303):
 *   opmode "RC": A is M x K row-major, B is K x N column-major;
 *   C is M x N column-major (ldC = M); FP32 accumulation.
 * Indices are int64.
 */
#ifndef KEBAB_KEBAB_H_
#define KEBAB_KEBAB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kebab_stream_t; /* same type as cudaStream_t */

typedef enum kebab_dtype {
  KEBAB_F16 = 0,  /* __half (IEEE binary16) */
  KEBAB_BF16 = 1, /* __nv_bfloat16 */
  KEBAB_F32 = 2   /* float: accepted by the dispatcher, rejected as ENOTSUP
                     exactly like baseline::gemm(const float*...) which prints
                     "not implemented" (cuda_gemm.cu:246-253) */
} kebab_dtype;

/* Status codes. */
#define KEBAB_OK 0
#define KEBAB_EINVAL 22     /* bad pointer, shape, opmode, alignment or version */
#define KEBAB_ENOTSUP 95    /* valid request this build does not implement */
#define KEBAB_ECUDA 1001    /* a CUDA runtime/driver call or launch failed */
#define KEBAB_ETIMEOUT 1002 /* a kernel's bounded wait expired (device status) */
#define KEBAB_ESPARSE 1003  /* input is not 2:4 sparse (pack step) */

/* Dense GEMM C = A * B through the version ladder.
 * Replaces baseline::gemm(const T* A, const T* B, T* C, int M, int N, int K,
 *   const char* opmode, int version, cudaStream_t stream)
 *   (kebab/lib/cuda/cuda_gemm.cu:112 for __half, :259 for __nv_bfloat16,
 *   :246 for float), returning a status instead of printing and returning.
 * `version` is one of the B200 rungs (1, 101..106, 120) or a reference
 * version id (2..20, 41), which maps to the B200 rung with the same idea
 * (kebab_version_name() tells which). opmode NULL means "RC". */
int kebab_gemm(kebab_dtype dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
               const char* opmode, int version, kebab_stream_t stream);

/* Name of a version, as used in CSV variant names.
 * Replaces baseline::gemm_cuda_version_feature_name(int)
 *   (kebab/lib/cuda/cuda_gemm.cu:81-106); "unknown" for unknown ids. */
const char* kebab_version_name(int version);

/* The B200 rung a version id resolves to for (dtype, M, N, K), after the
 * reference-id mapping and, for 120, the decomposition heuristic (the role
 * of the reference's v20 dispatcher, cuda_gemm.cu:25-77,211-230). Returns the
 * rung id, or a negative KEBAB_* code. */
int kebab_resolve_version(int version, kebab_dtype dtype, int64_t M, int64_t N, int64_t K);

/* Fills `out` with the implemented version ids (up to `cap`); returns count. */
int kebab_list_versions(int* out, int cap);

/* Message of the last failure on this thread ("" if none). No reference
 * counterpart: the reference prints to stderr (cuda_gemm.cu:115-122). */
const char* kebab_last_error(void);

/* Reads (and with clear != 0 resets) the device status word that kernels
 * set when a bounded wait expires. Synchronizes `stream` first. Returns
 * KEBAB_OK if the word was zero, KEBAB_ETIMEOUT otherwise; *code (optional)
 * receives the raw word (bits 0..7 class, 8..15 wait site, 16..31 block).
 * No reference counterpart: the reference's waits spin forever
 * (cuda_gemm_v10_*:196-209). */
int kebab_device_status(kebab_stream_t stream, uint32_t* code, int clear);

/* Per-wait budget of every kernel launched afterwards (default 2000 ms, or
 * the KEBAB_WAIT_TIMEOUT_MS environment variable). */
int kebab_set_wait_timeout_us(uint64_t timeout_us);

/* Arms a clock probe for the next tcgen05 GEMM launch (dense rungs 103-112,
 * 141, and the 2:4 sparse GEMM) made by this host thread: thread 0 of every
 * CTA of that launch writes four uint64 at buf[4 * cta]: the SM cycle counter
 * and the global nanosecond timer at entry, then both again at exit.
 * Cycles / nanoseconds is the SM clock in GHz that CTA ran at. `buf` is a
 * device buffer of 4 * max_ctas uint64; a launch with more CTAs than that
 * leaves the probe armed and writes nothing. (NULL, 0) disarms. No
 * reference counterpart: measurement support for the roofline. */
int kebab_clock_probe(void* buf, int64_t max_ctas);

/* Launches a one-warp kernel that waits on an mbarrier nobody arrives at,
 * with a budget of `timeout_us`; the wait expires and the kernel returns.
 * Exercises the timeout path without faulting or hanging the GPU. Returns
 * the status read back afterwards (KEBAB_ETIMEOUT when it works) and clears
 * it. */
int kebab_probe_wait_timeout(kebab_stream_t stream, uint64_t timeout_us);

/* Stream-K GEMM (rung 109's kernel: CTA pairs, RC, column-major C) that
 * allocates no device memory, for callers that cannot call cudaMalloc at that
 * point — a custom allocator or pool callback, a serving loop with a fixed
 * memory budget, a plugin host that forbids allocation after start-up. Its
 * scratch is a static device array present on every GPU that loads the
 * library: 160 partial-tile slots of 128 KiB (20 MiB) plus 2.5 KiB of flags;
 * a device whose grid needs more than 160 CTAs gets KEBAB_ENOTSUP. A
 * per-device set-up looks up the array's address and opts the kernels in; it
 * is also when the driver loads this code onto the device and commits the
 * 20 MiB, so it is the one step that may allocate. It runs on the first call
 * on a device, or alone when called with null A, B, C and M = N = K = 0 (then
 * it returns KEBAB_OK and launches nothing): make it before the code that must
 * not allocate and before any stream capture. Later calls allocate nothing.
 * All calls share the array, so calls that overlap on the GPU race.
 * kebab_shutdown() forgets the set-up. No counterpart in the reference. */
int kebab_gemm_streamk_noalloc(kebab_dtype dtype, const void* A, const void* B, void* C, int64_t M, int64_t N,
                               int64_t K, kebab_stream_t stream);

/* Releases cached tensor maps and per-device state. Replaces nothing: the
 * reference's function-static caches are never freed (cuda_gemm_v10_*:499). */
void kebab_shutdown(void);

#ifdef __cplusplus
}
#endif
#endif /* KEBAB_KEBAB_H_ */
