// libfmha_bwd_fp16.so: the fp16 attention-backward C-ABI.
// Drop-in for fmha_bwd_full_fp16, src/fmha_bwd_kernels_fp16.hip:235-280.
#include <cuda_fp16.h>

#include "fmha_bwd_common_abi.cuh"
#include "fmha_bwd_launch.cuh"

using fp16 = __half;

extern "C" {

FMHA_API void fmha_bwd_full_fp16(fp16* dQ, fp16* dK, fp16* dV, const fp16* Q, const fp16* K, const fp16* V,
                        const fp16* P, const fp16* dO, int M, int N, int K_dim, int total_heads) {
  fmha_sm100::run_backward<fp16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                 cudaStreamLegacy, /*sync=*/true);
}

FMHA_API int fmha_bwd_full_fp16_stream(fp16* dQ, fp16* dK, fp16* dV, const fp16* Q, const fp16* K,
                              const fp16* V, const fp16* P, const fp16* dO, int M, int N,
                              int K_dim, int total_heads, cudaStream_t stream) {
  return fmha_sm100::run_backward<fp16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false);
}

FMHA_API int fmha_bwd_full_fp16_delta(fp16* dQ, fp16* dK, fp16* dV, const fp16* Q, const fp16* K,
                                      const fp16* V, const fp16* P, const fp16* dO, const float* Dsum,
                                      int M, int N, int K_dim, int total_heads, cudaStream_t stream) {
  return fmha_sm100::run_backward<fp16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false, nullptr, Dsum, /*need_given_d=*/true);
}

FMHA_API int fmha_bwd_full_fp16_stream_events(fp16* dQ, fp16* dK, fp16* dV, const fp16* Q, const fp16* K,
                             const fp16* V, const fp16* P, const fp16* dO, int M, int N, int K_dim,
                             int total_heads, cudaStream_t stream, cudaEvent_t const* events) {
  return fmha_sm100::run_backward<fp16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false, events);
}

}  // extern "C"
