// libfmha_bwd_fp16.so: the fp16 attention-backward C-ABI.
// Drop-in for fmha_bwd_full_fp16, src/fmha_bwd_kernels_fp16.hip:235-280.
#include <cuda_fp16.h>

#include "fmha_bwd_common_abi.cuh"
#include "fmha_bwd_launch.cuh"
#include "fmha_bwd_stages.cuh"
#include "fmha_bwd_lse.cuh"

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

// ---- recompute-P entry: P = exp(scale Q K^T - LSE) is formed on chip; D =
// rowsum(dO * O). Stream-ordered; returns 0 or an error code.
FMHA_API int fmha_bwd_full_fp16_lse(fp16* dQ, fp16* dK, fp16* dV, const fp16* Q, const fp16* K, const fp16* V,
                      const fp16* O, const fp16* dO, const float* LSE, int M, int N, int K_dim,
                      int total_heads, float softmax_scale, cudaStream_t stream) {
  return fmha_sm100::run_backward_lse<fp16>(dQ, dK, dV, Q, K, V, O, dO, LSE, M, N, K_dim, total_heads,
                                          softmax_scale, stream);
}

// ---- stage hooks (replace the reference's test_* wrappers, src/fmha_bwd_kernels_fp16.hip:284-314; C++ linkage there,
// C linkage here).
// Each launches one stage on the legacy default stream and returns without
// waiting, like the reference; errors go to fmha_bwd_last_error().

FMHA_API void test_dp_kernel_fp16(const fp16* dO, const fp16* V, fp16* dP, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<fp16>(fmha_sm100::Stage::kDp, dO, V, dP, M, N, K_dim, total_heads);
}

FMHA_API void test_softmax_bwd_kernel_fp16(const fp16* P, const fp16* dP, fp16* dS, int M, int N,
                                        int total_heads) {
  fmha_sm100::run_stage_softmax_bwd<fp16>(P, dP, dS, M, N, total_heads);
}

FMHA_API void test_dq_kernel_fp16(const fp16* dS, const fp16* K, fp16* dQ, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<fp16>(fmha_sm100::Stage::kDq, dS, K, dQ, M, N, K_dim, total_heads);
}

FMHA_API void test_dk_kernel_fp16(const fp16* dS, const fp16* Q, fp16* dK, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<fp16>(fmha_sm100::Stage::kDk, dS, Q, dK, M, N, K_dim, total_heads);
}

FMHA_API void test_dv_kernel_fp16(const fp16* P, const fp16* dO, fp16* dV, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<fp16>(fmha_sm100::Stage::kDv, P, dO, dV, M, N, K_dim, total_heads);
}

}  // extern "C"
