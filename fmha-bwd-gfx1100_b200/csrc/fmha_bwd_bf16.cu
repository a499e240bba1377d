// libfmha_bwd_bf16.so: the bf16 attention-backward C-ABI.
// Drop-in for fmha_bwd_full_py, src/fmha_bwd_kernels.hip:474-523.
#include <cuda_bf16.h>

#include "fmha_bwd_common_abi.cuh"
#include "fmha_bwd_launch.cuh"

using bf16 = __nv_bfloat16;

extern "C" {

FMHA_API void fmha_bwd_full_py(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K, const bf16* V,
                      const bf16* P, const bf16* dO, int M, int N, int K_dim, int total_heads) {
  fmha_sm100::run_backward<bf16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                 cudaStreamLegacy, /*sync=*/true);
}

FMHA_API int fmha_bwd_full_stream(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K,
                         const bf16* V, const bf16* P, const bf16* dO, int M, int N, int K_dim,
                         int total_heads, cudaStream_t stream) {
  return fmha_sm100::run_backward<bf16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false);
}

FMHA_API int fmha_bwd_full_stream_events(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K,
                             const bf16* V, const bf16* P, const bf16* dO, int M, int N, int K_dim,
                             int total_heads, cudaStream_t stream, cudaEvent_t const* events) {
  return fmha_sm100::run_backward<bf16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false, events);
}

}  // extern "C"
