// libfmha_bwd_bf16.so: the bf16 attention-backward C-ABI.
// Drop-in for fmha_bwd_full_py, src/fmha_bwd_kernels.hip:474-523.
#include <cuda_bf16.h>

#include "fmha_bwd_common_abi.cuh"
#include "fmha_bwd_launch.cuh"
#include "fmha_bwd_stages.cuh"
#include "fmha_bwd_lse.cuh"

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------ no-alloc entry
// fmha_bwd_full_noalloc runs the same two kernels with the rowsum scratch
// (D, one float per query row and head) and the wait-status slot taken from
// the file-scope device arrays below instead of from cudaMalloc'd /
// cudaHostAlloc'd memory. It serves callers that must not allocate device
// memory from inside a library call.
namespace {

// Upper bound on total_heads * M for the no-alloc entry point: 2^20 rows of
// fp32 D, 4 MiB of device memory per device that loads this library.
constexpr size_t kNoAllocMaxRows = size_t(1) << 20;

static __device__ __align__(256) float g_noalloc_dsum[kNoAllocMaxRows];
static __device__ __align__(256) fmha_sm100::KernelStatus g_noalloc_status;

constexpr int kNoAllocMaxDevices = 64;

struct NoAllocSlot {
  float* dsum = nullptr;
  fmha_sm100::KernelStatus* status = nullptr;
  bool ready = false;
};

NoAllocSlot g_noalloc_slots[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current: device addresses of the two
// scratch arrays, and the kernels' shared-memory attributes. A set-up that
// fails is not remembered: the next call on that device tries again.
// Returns cudaSuccess or the error of the failed step.
cudaError_t noalloc_setup(int device, NoAllocSlot& out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  NoAllocSlot& s = g_noalloc_slots[device];
  if (!s.ready) {
    float* dsum = nullptr;
    fmha_sm100::KernelStatus* status = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&dsum), g_noalloc_dsum);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_noalloc_status);
    if (e == cudaSuccess) {
      fmha_sm100::set_kernel_attrs<bf16>();
      e = cudaGetLastError();
    } else {
      cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
    s.dsum = dsum;
    s.status = status;
    s.ready = true;
  }
  out = s;
  return cudaSuccess;
}

}  // namespace

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

FMHA_API int fmha_bwd_full_delta(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K,
                                 const bf16* V, const bf16* P, const bf16* dO, const float* Dsum,
                                 int M, int N, int K_dim, int total_heads, cudaStream_t stream) {
  return fmha_sm100::run_backward<bf16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false, nullptr, Dsum, /*need_given_d=*/true);
}

FMHA_API int fmha_bwd_full_stream_events(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K,
                             const bf16* V, const bf16* P, const bf16* dO, int M, int N, int K_dim,
                             int total_heads, cudaStream_t stream, cudaEvent_t const* events) {
  return fmha_sm100::run_backward<bf16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads,
                                        stream, /*sync=*/false, events);
}

// No counterpart in the reference. Same operation and preconditions as
// fmha_bwd_full_stream, plus total_heads * M <= kNoAllocMaxRows; allocates
// nothing. Enqueues on `stream`, waits for it, and returns 0 or an error code.
// The first call on a device looks up the scratch arrays' addresses (module
// load included). Every call shares the one scratch: calls that overlap on the GPU (other
// streams, other host threads) race.
FMHA_API int fmha_bwd_full_noalloc(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K,
                                   const bf16* V, const bf16* P, const bf16* dO, int M, int N,
                                   int K_dim, int total_heads, cudaStream_t stream) {
  using namespace fmha_sm100;
  int rc = check_args(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads);
  if (rc != kOk) return rc;
  const size_t rows = static_cast<size_t>(total_heads) * static_cast<size_t>(M);
  if (rows > kNoAllocMaxRows)
    return set_error(kErrInvalidArgument,
                     "total_heads*M = %zu exceeds the no-alloc scratch limit of %zu rows", rows,
                     kNoAllocMaxRows);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kErrLaunch, "no current CUDA device");
  }
  if (device < 0 || device >= kNoAllocMaxDevices)
    return set_error(kErrInvalidArgument, "device ordinal %d beyond %d", device, kNoAllocMaxDevices);
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0)
    return set_error(kErrUnsupportedDevice, "device %d is sm_%d%d; this library needs sm_100", device,
                     major, minor);
  NoAllocSlot slot;
  const cudaError_t se = noalloc_setup(device, slot);
  if (se != cudaSuccess)
    return set_error(kErrLaunch, "no-alloc scratch set-up failed: %s", cudaGetErrorString(se));

  // The status slot must start at zero; D needs no clearing (the dQ kernel
  // writes every row that the dK/dV kernel reads, earlier on the same stream).
  cudaError_t e = cudaMemsetAsync(slot.status, 0, sizeof(KernelStatus), stream);
  if (e != cudaSuccess) return set_error(kErrLaunch, "status reset failed: %s", cudaGetErrorString(e));
  rc = enqueue_backward<bf16>(dQ, dK, dV, Q, K, V, P, dO, M, N, K_dim, total_heads, slot.dsum,
                              slot.status, stream, nullptr);
  if (rc != kOk) return rc;
  // read the status word on the caller's stream, then wait for that stream
  // alone (no device-wide synchronisation)
  KernelStatus st{};
  e = cudaMemcpyAsync(&st, slot.status, sizeof(KernelStatus), cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return set_error(kErrLaunch, "status read failed: %s", cudaGetErrorString(e));
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return set_error(kErrLaunch, "kernel failed: %s", cudaGetErrorString(e));
  if (st.code != 0)
    return set_error(kErrDeviceTimeout, "in-kernel wait gave up (code %d, site %d, block %d)",
                     st.code, st.where, st.block);
  return set_error(kOk, "");
}

// ---- recompute-P entry: P = exp(scale Q K^T - LSE) is formed on chip; D =
// rowsum(dO * O). Stream-ordered; returns 0 or an error code.
FMHA_API int fmha_bwd_full_lse(bf16* dQ, bf16* dK, bf16* dV, const bf16* Q, const bf16* K, const bf16* V,
                      const bf16* O, const bf16* dO, const float* LSE, int M, int N, int K_dim,
                      int total_heads, float softmax_scale, cudaStream_t stream) {
  return fmha_sm100::run_backward_lse<bf16>(dQ, dK, dV, Q, K, V, O, dO, LSE, M, N, K_dim, total_heads,
                                          softmax_scale, stream);
}

// ---- stage hooks (replace the reference's test_* wrappers, src/fmha_bwd_kernels.hip:525-560).
// Each launches one stage on the legacy default stream and returns without
// waiting, like the reference; errors go to fmha_bwd_last_error().

FMHA_API void test_dp_kernel(const bf16* dO, const bf16* V, bf16* dP, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<bf16>(fmha_sm100::Stage::kDp, dO, V, dP, M, N, K_dim, total_heads);
}

FMHA_API void test_softmax_bwd_kernel(const bf16* P, const bf16* dP, bf16* dS, int M, int N,
                                        int total_heads) {
  fmha_sm100::run_stage_softmax_bwd<bf16>(P, dP, dS, M, N, total_heads);
}

FMHA_API void test_dq_kernel(const bf16* dS, const bf16* K, bf16* dQ, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<bf16>(fmha_sm100::Stage::kDq, dS, K, dQ, M, N, K_dim, total_heads);
}

FMHA_API void test_dk_kernel(const bf16* dS, const bf16* Q, bf16* dK, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<bf16>(fmha_sm100::Stage::kDk, dS, Q, dK, M, N, K_dim, total_heads);
}

FMHA_API void test_dv_kernel(const bf16* P, const bf16* dO, bf16* dV, int M, int N, int K_dim,
                               int total_heads) {
  fmha_sm100::run_stage_gemm<bf16>(fmha_sm100::Stage::kDv, P, dO, dV, M, N, K_dim, total_heads);
}

}  // extern "C"
