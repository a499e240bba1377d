/* C-ABI of the B200 (sm_100a) attention-backward libraries.
 *
 *   build/libfmha_bwd_bf16.so  exports the bf16 entry points
 *   build/libfmha_bwd_fp16.so  exports the fp16 entry points
 *
 * Both libraries are drop-in replacements for the reference's
 * build/libfmha_bwd_bf16.so / build/libfmha_bwd_fp16.so: the ctypes host in
 * benchmark_pytorch_final.py:30-37 loads them and calls them unchanged.
 *
 * Semantics (no softmax scale; src/kernel/correct/cpu_reference.hpp:30-40,
 * :74-126), for every head h:
 *   dP = dO V^T;  D = rowsum(P * dP);  dS = P * (dP - D)
 *   dQ = dS K;    dK = dS^T Q;          dV = P^T dO
 * Layout per head h (row-major, heads contiguous): Q, dO, dQ at h*M*K_dim;
 * K, V, dK, dV at h*N*K_dim; P at h*M*N (src/fmha_bwd_kernels.hip:72-74).
 * Inputs are read only; dQ, dK and dV are fully overwritten.
 *
 * Preconditions (checked before anything is launched; on failure nothing is
 * written, a message goes to stderr and fmha_bwd_last_error() is non-zero):
 *   M, N, total_heads > 0; K_dim is 64 or 128; total_heads <= 65535;
 *   N % 8 == 0 (each P row starts on a 16-byte boundary);
 *   every pointer is 16-byte aligned device memory of the current device,
 *   which must be an sm_100 GPU.
 *
 * Storage types are 16-bit; the C side sees them as uint16_t.
 */
#ifndef FMHA_BWD_B200_H_
#define FMHA_BWD_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t fmha_bf16_t; /* bfloat16 bits */
typedef uint16_t fmha_fp16_t; /* IEEE half bits */
typedef struct CUstream_st* fmha_stream_t; /* cudaStream_t */

/* Error codes (fmha_bwd_last_error). */
enum {
  FMHA_BWD_OK = 0,
  FMHA_BWD_ERR_INVALID_ARGUMENT = 1,
  FMHA_BWD_ERR_MISALIGNED = 2,
  FMHA_BWD_ERR_UNSUPPORTED_DEVICE = 3,
  FMHA_BWD_ERR_OUT_OF_MEMORY = 4,
  FMHA_BWD_ERR_LAUNCH = 5,
  FMHA_BWD_ERR_DEVICE_TIMEOUT = 6,
  FMHA_BWD_ERR_NO_DRIVER = 7
};

/* ---- libfmha_bwd_bf16.so ------------------------------------------------ */

/* Replaces fmha_bwd_full_py, src/fmha_bwd_kernels.hip:474-477 (bf16).
 * Launches on the legacy default stream and returns after that stream has
 * finished, like the reference (which ends with hipDeviceSynchronize, :520). */
void fmha_bwd_full_py(fmha_bf16_t* dQ, fmha_bf16_t* dK, fmha_bf16_t* dV,
                      const fmha_bf16_t* Q, const fmha_bf16_t* K,
                      const fmha_bf16_t* V, const fmha_bf16_t* P,
                      const fmha_bf16_t* dO, int M, int N, int K_dim,
                      int total_heads);

/* Stream-ordered variant (the reference's stale header imagines a stream
 * argument for fmha_bwd_full, src/fmha_bwd_kernels.hpp:60-65). Enqueues the
 * work on `stream` and returns at once with 0, or an error code if the call
 * was rejected before launch. Calls on different streams of one device must
 * not overlap: they share the device's workspace. */
int fmha_bwd_full_stream(fmha_bf16_t* dQ, fmha_bf16_t* dK, fmha_bf16_t* dV,
                         const fmha_bf16_t* Q, const fmha_bf16_t* K,
                         const fmha_bf16_t* V, const fmha_bf16_t* P,
                         const fmha_bf16_t* dO, int M, int N, int K_dim,
                         int total_heads, fmha_stream_t stream);

/* Profiling variant of fmha_bwd_full_stream: additionally records the four
 * CUDA events in `events` (cudaEvent_t[4], entries may be NULL) on `stream`:
 * [0] before the query-major dQ kernel, [1] between it and the key-major
 * dK/dV kernel, [2] and [3] after the dK/dV kernel, so a caller can time each
 * kernel inside a run.
 * No counterpart in the reference. */
int fmha_bwd_full_stream_events(fmha_bf16_t* dQ, fmha_bf16_t* dK,
                                fmha_bf16_t* dV, const fmha_bf16_t* Q,
                                const fmha_bf16_t* K, const fmha_bf16_t* V,
                                const fmha_bf16_t* P, const fmha_bf16_t* dO,
                                int M, int N, int K_dim, int total_heads,
                                fmha_stream_t stream, void* const* events);

/* Precomputed-rowsum variant of fmha_bwd_full_stream (the "accept a
 * precomputed D" extension the reference's path lacks; no reference
 * counterpart). Dsum[h * M + m] = sum_n P[h,m,n] * dP[h,m,n] in fp32, i.e.
 * rowsum(dO * O) when O = P V is the forward output, supplied by the caller
 * (float-aligned device memory, read only; 2 if misaligned). The dQ kernel then skips its
 * own rowsum and the extra P K accumulation (5 instead of 6 GEMM-sized MMA
 * passes). Stream-ordered; returns 0 or an error code (1 if Dsum is null). */
int fmha_bwd_full_delta(fmha_bf16_t* dQ, fmha_bf16_t* dK, fmha_bf16_t* dV,
                        const fmha_bf16_t* Q, const fmha_bf16_t* K,
                        const fmha_bf16_t* V, const fmha_bf16_t* P,
                        const fmha_bf16_t* dO, const float* Dsum, int M, int N,
                        int K_dim, int total_heads, fmha_stream_t stream);

/* Recompute-P variant (the reference's path reads a materialised P; this is
 * the "produce P on the fly from Q, K and the row log-sum-exp" extension, no
 * reference counterpart). Per head: O [M][K_dim] is the forward output and
 * LSE [M] (fp32, 4-byte aligned) holds log sum_n exp(softmax_scale Q_m.K_n).
 * The kernels form P = exp(softmax_scale Q K^T - LSE) on chip and return the
 * gradients of the scaled-score attention:
 *   D = rowsum(dO * O), dS = P * (dO V^T - D),
 *   dQ = softmax_scale dS K, dK = softmax_scale dS^T Q, dV = P^T dO.
 * With softmax_scale = 1 and O = P V this equals fmha_bwd_full_py on that P,
 * with no M x N buffer anywhere. N needs no alignment (no P rows are read);
 * other preconditions as fmha_bwd_full_py; softmax_scale > 0 and finite.
 * Stream-ordered; returns 0 or an error code. */
int fmha_bwd_full_lse(fmha_bf16_t* dQ, fmha_bf16_t* dK, fmha_bf16_t* dV,
                      const fmha_bf16_t* Q, const fmha_bf16_t* K,
                      const fmha_bf16_t* V, const fmha_bf16_t* O,
                      const fmha_bf16_t* dO, const float* LSE, int M, int N,
                      int K_dim, int total_heads, float softmax_scale,
                      fmha_stream_t stream);

/* No counterpart in the reference. Allocation-free variant of
 * fmha_bwd_full_stream: the fp32 rowsum scratch D (total_heads * M floats)
 * and the wait-status slot live in file-scope __device__ arrays of the
 * library instead of cudaMalloc / cudaHostAlloc memory, so the call makes no
 * allocation of any kind. Limit: total_heads * M <= 1048576 (4 MiB of
 * scratch); larger calls return FMHA_BWD_ERR_INVALID_ARGUMENT before any
 * launch. Enqueues on `stream`, waits for that stream and returns 0 or an
 * error code (in-kernel wait timeouts included). The first call on a device
 * looks up the scratch addresses (cudaGetSymbolAddress, which loads the
 * module). All calls share the one scratch: calls that overlap on the GPU
 * race. */
int fmha_bwd_full_noalloc(fmha_bf16_t* dQ, fmha_bf16_t* dK, fmha_bf16_t* dV,
                          const fmha_bf16_t* Q, const fmha_bf16_t* K,
                          const fmha_bf16_t* V, const fmha_bf16_t* P,
                          const fmha_bf16_t* dO, int M, int N, int K_dim,
                          int total_heads, fmha_stream_t stream);

/* Stage hooks (replace the reference's test_* wrappers,
 * src/fmha_bwd_kernels.hip:525-560). Each runs one stage of the backward as
 * its own launch with its 16-bit intermediate in global memory ([H][M][N]
 * for dP and dS), on the legacy default stream, and returns without waiting,
 * as the reference does. Same layout and preconditions as fmha_bwd_full_py
 * (N % 8 == 0, K_dim 64 or 128, 16-byte aligned pointers); a rejected call
 * launches nothing and sets fmha_bwd_last_error(); in-kernel wait timeouts
 * are read with fmha_bwd_poll_device_status() after the stream finished.
 * The production entry points never use them (dP and dS stay on chip). */

/* dP = dO V^T (src/fmha_bwd_kernels.hip:525-529). */
void test_dp_kernel(const fmha_bf16_t* dO, const fmha_bf16_t* V, fmha_bf16_t* dP,
                    int M, int N, int K_dim, int total_heads);

/* dS = P * (dP - rowsum(P * dP)), rowsum in fp32 (:531-536). */
void test_softmax_bwd_kernel(const fmha_bf16_t* P, const fmha_bf16_t* dP,
                             fmha_bf16_t* dS, int M, int N, int total_heads);

/* dQ = dS K (:538-542). */
void test_dq_kernel(const fmha_bf16_t* dS, const fmha_bf16_t* K, fmha_bf16_t* dQ,
                    int M, int N, int K_dim, int total_heads);

/* dK = dS^T Q (:544-548). */
void test_dk_kernel(const fmha_bf16_t* dS, const fmha_bf16_t* Q, fmha_bf16_t* dK,
                    int M, int N, int K_dim, int total_heads);

/* dV = P^T dO (:550-554; the reference names the last size BK_dim). */
void test_dv_kernel(const fmha_bf16_t* P, const fmha_bf16_t* dO, fmha_bf16_t* dV,
                    int M, int N, int K_dim, int total_heads);

/* ---- libfmha_bwd_fp16.so ------------------------------------------------ */

/* Replaces fmha_bwd_full_fp16, src/fmha_bwd_kernels_fp16.hip:236-238. */
void fmha_bwd_full_fp16(fmha_fp16_t* dQ, fmha_fp16_t* dK, fmha_fp16_t* dV,
                        const fmha_fp16_t* Q, const fmha_fp16_t* K,
                        const fmha_fp16_t* V, const fmha_fp16_t* P,
                        const fmha_fp16_t* dO, int M, int N, int K_dim,
                        int total_heads);

/* fp16 stream-ordered variant, as fmha_bwd_full_stream. */
int fmha_bwd_full_fp16_stream(fmha_fp16_t* dQ, fmha_fp16_t* dK,
                              fmha_fp16_t* dV, const fmha_fp16_t* Q,
                              const fmha_fp16_t* K, const fmha_fp16_t* V,
                              const fmha_fp16_t* P, const fmha_fp16_t* dO,
                              int M, int N, int K_dim, int total_heads,
                              fmha_stream_t stream);

/* fp16 precomputed-rowsum variant, as fmha_bwd_full_delta. */
int fmha_bwd_full_fp16_delta(fmha_fp16_t* dQ, fmha_fp16_t* dK, fmha_fp16_t* dV,
                             const fmha_fp16_t* Q, const fmha_fp16_t* K,
                             const fmha_fp16_t* V, const fmha_fp16_t* P,
                             const fmha_fp16_t* dO, const float* Dsum, int M,
                             int N, int K_dim, int total_heads,
                             fmha_stream_t stream);

/* fp16 recompute-P variant, as fmha_bwd_full_lse. */
int fmha_bwd_full_fp16_lse(fmha_fp16_t* dQ, fmha_fp16_t* dK, fmha_fp16_t* dV,
                           const fmha_fp16_t* Q, const fmha_fp16_t* K,
                           const fmha_fp16_t* V, const fmha_fp16_t* O,
                           const fmha_fp16_t* dO, const float* LSE, int M, int N,
                           int K_dim, int total_heads, float softmax_scale,
                           fmha_stream_t stream);

/* fp16 profiling variant, as fmha_bwd_full_stream_events. */
int fmha_bwd_full_fp16_stream_events(fmha_fp16_t* dQ, fmha_fp16_t* dK,
                                     fmha_fp16_t* dV, const fmha_fp16_t* Q,
                                     const fmha_fp16_t* K, const fmha_fp16_t* V,
                                     const fmha_fp16_t* P, const fmha_fp16_t* dO,
                                     int M, int N, int K_dim, int total_heads,
                                     fmha_stream_t stream, void* const* events);

/* fp16 stage hooks, as the bf16 ones (src/fmha_bwd_kernels_fp16.hip:284-314,
 * where they have C++ linkage; here they are plain C symbols). */
void test_dp_kernel_fp16(const fmha_fp16_t* dO, const fmha_fp16_t* V, fmha_fp16_t* dP,
                         int M, int N, int K_dim, int total_heads);
void test_softmax_bwd_kernel_fp16(const fmha_fp16_t* P, const fmha_fp16_t* dP,
                                  fmha_fp16_t* dS, int M, int N, int total_heads);
void test_dq_kernel_fp16(const fmha_fp16_t* dS, const fmha_fp16_t* K, fmha_fp16_t* dQ,
                         int M, int N, int K_dim, int total_heads);
void test_dk_kernel_fp16(const fmha_fp16_t* dS, const fmha_fp16_t* Q, fmha_fp16_t* dK,
                         int M, int N, int K_dim, int total_heads);
void test_dv_kernel_fp16(const fmha_fp16_t* P, const fmha_fp16_t* dO, fmha_fp16_t* dV,
                         int M, int N, int K_dim, int total_heads);

/* ---- exported by both libraries ---------------------------------------- */

/* Additive to the reference (whose entry returns void and only prints on
 * allocation failure, src/fmha_bwd_kernels.hip:486-490): the code of the most
 * recent call in this process (FMHA_BWD_OK if it succeeded). For the stream
 * variants, in-kernel wait timeouts are reported by the next synchronous call
 * or by fmha_bwd_poll_device_status() after the stream has finished. */
int fmha_bwd_last_error(void);

/* Human-readable message for the most recent error ("" if none). */
const char* fmha_bwd_last_error_message(void);

/* Reads and clears the status slot of the current device (host-mapped
 * memory that the kernels write when an in-kernel wait runs out): 0 if every
 * wait of every call since the last poll completed, else
 * FMHA_BWD_ERR_DEVICE_TIMEOUT. Call after synchronising the stream. */
int fmha_bwd_poll_device_status(void);

/* No counterpart in the reference. Self-test of the bounded in-kernel waits:
 * launches one warp that waits on a barrier nothing arrives on, with a limit
 * of `timeout_ms` (1..10000). Returns FMHA_BWD_OK if the wait gave up, the
 * timeout was recorded in the status slot and the kernel exited normally (the
 * context stays usable); otherwise an error code. Synchronises the device. */
int fmha_bwd_selftest_wait_timeout(int timeout_ms);

/* No counterpart in the reference. Host-only, launches nothing: how a call
 * divides `items` work items of `len` steps each (query tiles for the dQ
 * kernel, key tiles for the dK/dV kernel, times total_heads) over `grid`
 * persistent CTAs. out[0] = items run whole, out[1] = parts each remaining
 * (tail) item is split into (1: none), out[2] = work units in all; a split
 * kernel is followed by a combine kernel. `allow` = 0 reports the plan of a
 * call without a partial-sum workspace (never split). Returns FMHA_BWD_OK,
 * or FMHA_BWD_ERR_INVALID_ARGUMENT for a null `out` or negative sizes. */
int fmha_bwd_work_units(int items, int grid, int len, int allow, int* out);

/* Upper bound, in milliseconds, on any single in-kernel wait (default 4000,
 * or FMHA_BWD_WAIT_TIMEOUT_MS). A wait that runs out sets the device status
 * word and the kernel drains and exits instead of hanging. 0 restores the
 * default. */
void fmha_bwd_set_wait_timeout_ms(int ms);

#ifdef __cplusplus
}
#endif

#endif /* FMHA_BWD_B200_H_ */
