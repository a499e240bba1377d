// Stage hooks: each stage of the attention backward as its own launch, with
// its 16-bit intermediate in global memory, for testing a stage in
// isolation. They replace the reference's test_* wrappers
// (src/fmha_bwd_kernels.hip:525-560, src/fmha_bwd_kernels_fp16.hip:285-314):
//
//   dp           dP = dO V^T                      [H][M][N]
//   softmax_bwd  dS = P * (dP - rowsum(P * dP))   [H][M][N]
//   dq           dQ = dS K                        [H][M][d]
//   dk           dK = dS^T Q                      [H][N][d]
//   dv           dV = P^T dO                      [H][N][d]
//
// The four products run on one tcgen05 GEMM kernel (stage_gemm_kernel),
// templated on the major-ness of its operands, so every operand is read by
// TMA straight from the caller's row-major buffers (a transposed operand is
// an MN-major UMMA operand, never an explicit transpose). The row reduction
// runs on stage_softmax_bwd_kernel (one CTA per row, fp32 sum).
//
// The production path (fmha_bwd_full_py) does not use these: it keeps dP and
// dS on chip. They exist for stage-level testing and debugging.
#pragma once

#include "fmha_bwd_launch.cuh"

namespace fmha_sm100 {

// ======================================================== stage_gemm_kernel
// C[h] (R x Cc, 16-bit, row-major) = sum_k A[h](r, k) B[h](k, c), fp32
// accumulation in TMEM. One CTA per 128 x kN output tile and head.
//   kAMN = false: A stored [R][Kc] (K-major); true: stored [Kc][R] (MN-major).
//   kBMN = false: B stored [Cc][Kc] (K-major); true: stored [Kc][Cc] (MN-major).
// The contraction runs in blocks of 64 through a kStages-deep ring of TMA
// tiles; out-of-range rows and columns are zero-filled by TMA, so ragged R,
// Cc and Kc need no special case on the load side.
struct StageGemmCfg {
  static constexpr int kStages = 3;
  static constexpr int kKBlock = 64;
  static constexpr int kABytes = kTile * kKBlock * 2;  // 16 KB
  static constexpr int kThreads = 128;
};

template <int kN>
struct StageGemmLayout {
  static constexpr int kBBytes = kN * StageGemmCfg::kKBlock * 2;
  static constexpr int kStageBytes = StageGemmCfg::kABytes + kBBytes;
  static constexpr int kTileBytes = StageGemmCfg::kStages * kStageBytes;
  static constexpr int kSmemBytes = kTileBytes + 128 + 1024;
  static_assert(kN == 64 || kN == 128, "output tile width");
};

template <typename T, int kN, bool kAMN, bool kBMN>
__global__ void __launch_bounds__(StageGemmCfg::kThreads)
    stage_gemm_kernel(const __grid_constant__ CUtensorMap tm_A, const __grid_constant__ CUtensorMap tm_B,
                      T* __restrict__ C, int R, int Cc, int Kc, KernelStatus* status,
                      uint64_t timeout_ns) {
  using L = StageGemmLayout<kN>;
  constexpr int S = StageGemmCfg::kStages;
  constexpr int kAB = StageGemmCfg::kABytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::kTileBytes);  // full[S], empty[S], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2 * S + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * kN;
  const int r0 = blockIdx.y * kTile;
  const int h = blockIdx.z;
  const int nkb = (Kc + StageGemmCfg::kKBlock - 1) / StageGemmCfg::kKBlock;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bar[s], 1);
      mbar_init(&bar[S + s], 1);
    }
    mbar_init(&bar[2 * S], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  WaitCtx ctx{abort_flag, timeout_ns};

  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_A);
      tma_prefetch_desc(&tm_B);
      const uint64_t pol = l2_policy_evict_normal();
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        if (kb >= S && !mbar_wait(&bar[S + s], ((kb / S) - 1) & 1, ctx, 60)) break;
        uint8_t* sa = smem + s * L::kStageBytes;
        uint8_t* sb = sa + kAB;
        const int k0 = kb * StageGemmCfg::kKBlock;
        mbar_arrive_expect_tx(&bar[s], L::kStageBytes);
        if constexpr (kAMN) {  // [Kc][R]: two 64-column boxes of 64 rows
          tma_load_3d(sa, &tm_A, &bar[s], r0, k0, h, pol);
          tma_load_3d(sa + kAB / 2, &tm_A, &bar[s], r0 + kBoxCols, k0, h, pol);
        } else {  // [R][Kc]: one 64-column box of 128 rows
          tma_load_3d(sa, &tm_A, &bar[s], k0, r0, h, pol);
        }
        if constexpr (kBMN) {  // [Kc][Cc]: kN / 64 boxes of 64 rows
#pragma unroll
          for (int b = 0; b < kN / kBoxCols; ++b)
            tma_load_3d(sb + b * (L::kBBytes * kBoxCols / kN), &tm_B, &bar[s], c0 + b * kBoxCols, k0, h, pol);
        } else {  // [Cc][Kc]: one 64-column box of kN rows
          tma_load_3d(sb, &tm_B, &bar[s], k0, c0, h, pol);
        }
        ++issued;
      }
      if (*abort_flag) {
        for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
          mbar_wait_drain(&bar[i % S], (i / S) & 1, timeout_ns);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: 4 MMAs (K = 16 each) per 64-wide contraction block
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16<Elem<T>::kBF16>(kTile, kN, kAMN, kBMN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&bar[s], (kb / S) & 1, ctx, 61)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
        const uint32_t sb = sa + kAB;
        // MN-major: 64-element MN blocks LBO apart, 16 contraction rows =
        // 2048 bytes per step. K-major: 32 bytes per step inside the row.
        const uint64_t da = kAMN ? make_sw128_desc(sa, kAB / 2, 1024) : make_sw128_desc(sa, 16, 1024);
        const uint64_t db = kBMN ? make_sw128_desc(sb, L::kBBytes * kBoxCols / kN, 1024)
                                 : make_sw128_desc(sb, 16, 1024);
#pragma unroll
        for (int k = 0; k < StageGemmCfg::kKBlock / 16; ++k) {
          const uint32_t step = kAMN ? 2048u * k : 32u * k;
          const uint32_t stepb = kBMN ? 2048u * k : 32u * k;
          umma_f16_ss(tmem, desc_advance(da, step), desc_advance(db, stepb), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&bar[S + s]);
      }
      // completion of every MMA issued above (also after an abort, so that
      // TMEM is not released under a running MMA)
      umma_commit(&bar[2 * S]);
    }
    __syncwarp();
  }

  // ---- epilogue: warp w reads TMEM lanes 32w..32w+31 = output rows
  {
    const bool done = mbar_wait(&bar[2 * S], 0, ctx, 62);
    __syncwarp();
    tc_fence_after();
    if (done && *abort_flag == 0) {
      const int r = r0 + 32 * warp + lane;
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
      T* out = C + (static_cast<int64_t>(h) * R + r) * Cc + c0;
#pragma unroll
      for (int x = 0; x < kN / 32; ++x) {
        uint32_t v[32];
        __syncwarp();  // .sync.aligned TMEM access: the warp reconverges after the
                       // row-guarded stores of the previous iteration
        tmem_load_32(lane_base + 32 * x, v);
        if (r < R) {
          if (c0 + 32 * x + 32 <= Cc) {
            store_row_32<T>(out + 32 * x, reinterpret_cast<const float*>(v));
          } else {
            // ragged column tail, in whole 16-byte chunks (Cc % 8 == 0)
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              if (c0 + 32 * x + 8 * y < Cc) {
                const float* f = reinterpret_cast<const float*>(v) + 8 * y;
                *reinterpret_cast<uint4*>(out + 32 * x + 8 * y) =
                    make_uint4(Elem<T>::pack(f[0], f[1]), Elem<T>::pack(f[2], f[3]),
                               Elem<T>::pack(f[4], f[5]), Elem<T>::pack(f[6], f[7]));
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) publish_failure(*abort_flag, status);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kN);
  }
}

// ================================================= stage_softmax_bwd_kernel
// One CTA per (row m, head h): D = sum_n P dP in fp32, then
// dS = P (dP - D) rounded to 16-bit (src/fmha_bwd_kernels.hip:54-102 computes
// the same per row; src/kernel/correct/cpu_reference.hpp:30-40). Rows are
// read in 16-byte chunks (N % 8 == 0); the second pass re-reads the row from
// L1/L2.
constexpr int kSoftmaxThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kSoftmaxThreads)
    stage_softmax_bwd_kernel(const T* __restrict__ P, const T* __restrict__ dP, T* __restrict__ dS,
                             int M, int N) {
  __shared__ float partial[kSoftmaxThreads / 32];
  const int64_t row = static_cast<int64_t>(blockIdx.y) * M + blockIdx.x;
  const uint4* p4 = reinterpret_cast<const uint4*>(P + row * N);
  const uint4* g4 = reinterpret_cast<const uint4*>(dP + row * N);
  uint4* s4 = reinterpret_cast<uint4*>(dS + row * N);
  const int chunks = N / 8;
  float acc = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kSoftmaxThreads) {
    const uint4 pv = __ldg(p4 + c), gv = __ldg(g4 + c);
    const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 p = Elem<T>::unpack(pw[t]), g = Elem<T>::unpack(gw[t]);
      acc = fmaf(p.x, g.x, acc);
      acc = fmaf(p.y, g.y, acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = acc;
  __syncthreads();
  float D = 0.f;
#pragma unroll
  for (int w = 0; w < kSoftmaxThreads / 32; ++w) D += partial[w];
  for (int c = threadIdx.x; c < chunks; c += kSoftmaxThreads) {
    const uint4 pv = __ldg(p4 + c), gv = __ldg(g4 + c);
    const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 p = Elem<T>::unpack(pw[t]), g = Elem<T>::unpack(gw[t]);
      o[t] = Elem<T>::pack(p.x * (g.x - D), p.y * (g.y - D));
    }
    s4[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ================================================================ host side
enum class Stage { kDp, kDq, kDk, kDv };

template <typename T>
void set_stage_attrs() {
  cudaFuncSetAttribute(stage_gemm_kernel<T, 128, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       StageGemmLayout<128>::kSmemBytes);
  cudaFuncSetAttribute(stage_gemm_kernel<T, 128, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       StageGemmLayout<128>::kSmemBytes);
  cudaFuncSetAttribute(stage_gemm_kernel<T, 64, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       StageGemmLayout<64>::kSmemBytes);
  cudaFuncSetAttribute(stage_gemm_kernel<T, 128, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       StageGemmLayout<128>::kSmemBytes);
  cudaFuncSetAttribute(stage_gemm_kernel<T, 64, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       StageGemmLayout<64>::kSmemBytes);
}

// Device checks shared by the stage hooks; returns the status slot of the
// current device (nullptr, error recorded, on failure).
template <typename T>
KernelStatus* stage_prepare() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    set_error(kErrLaunch, "no current CUDA device");
    return nullptr;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0) {
    set_error(kErrUnsupportedDevice, "device %d is sm_%d%d; this library needs sm_100", device, major, minor);
    return nullptr;
  }
  std::lock_guard<std::mutex> g(ws_mutex());
  DeviceWorkspace& w = ws_map()[device];
  if (!ensure_status_slot(device, w)) return nullptr;
  static std::once_flag once[64];
  if (device < 64) std::call_once(once[device], [] { set_stage_attrs<T>(); });
  else set_stage_attrs<T>();
  return w.host_status_dev;
}

// One GEMM stage on the legacy default stream (the reference's test_*
// wrappers launch on stream 0 and do not synchronise). `a` and `b` are the
// two inputs in the reference's argument order; `c` is the output.
template <typename T>
int run_stage_gemm(Stage st, const T* a, const T* b, T* c, int M, int N, int D, int H) {
  if (!a || !b || !c) return set_error(kErrInvalidArgument, "null pointer argument");
  if (M <= 0 || N <= 0 || H <= 0 || D <= 0)
    return set_error(kErrInvalidArgument, "sizes must be positive (M=%d N=%d K_dim=%d heads=%d)", M, N, D, H);
  if (D != 64 && D != 128) return set_error(kErrInvalidArgument, "K_dim=%d unsupported (64 or 128)", D);
  if (H > 65535) return set_error(kErrInvalidArgument, "total_heads=%d exceeds 65535", H);
  if (N % 8 != 0)
    return set_error(kErrMisaligned, "N=%d: [M][N] rows must be a multiple of 16 bytes (N %% 8 == 0)", N);
  if (!aligned16(a) || !aligned16(b) || !aligned16(c))
    return set_error(kErrMisaligned, "every buffer must be 16-byte aligned");
  const int out_rows = (st == Stage::kDk || st == Stage::kDv) ? N : M;
  if ((out_rows + kTile - 1) / kTile > 65535)
    return set_error(kErrInvalidArgument, "%d output rows exceed the grid limit", out_rows);
  KernelStatus* status = stage_prepare<T>();
  if (!status) return error_state().code.load();
  if (!encode_fn()) return set_error(kErrNoDriver, "cuTensorMapEncodeTiled is unavailable");
  constexpr bool kBF16 = Elem<T>::kBF16;
  const uint64_t tmo = effective_timeout_ns();
  CUtensorMap mA, mB;
  bool ok = false;
  dim3 grid;
  const dim3 block(StageGemmCfg::kThreads);
  cudaStream_t stream = cudaStreamLegacy;
  switch (st) {
    case Stage::kDp:  // dP[M][N] = dO[M][d] . V[N][d]^T: both K-major (K = d)
      ok = encode_map(&mA, kBF16, a, D, M, H, kTile) && encode_map(&mB, kBF16, b, D, N, H, 128);
      if (!ok) break;
      grid = dim3((N + 127) / 128, (M + kTile - 1) / kTile, H);
      stage_gemm_kernel<T, 128, false, false><<<grid, block, StageGemmLayout<128>::kSmemBytes, stream>>>(
          mA, mB, c, M, N, D, status, tmo);
      break;
    case Stage::kDq:  // dQ[M][d] = dS[M][N] . K[N][d]: A K-major (K = N), B MN-major
      ok = encode_map(&mA, kBF16, a, N, M, H, kTile) && encode_map(&mB, kBF16, b, D, N, H, 64);
      if (!ok) break;
      grid = dim3(1, (M + kTile - 1) / kTile, H);
      if (D == 128)
        stage_gemm_kernel<T, 128, false, true><<<grid, block, StageGemmLayout<128>::kSmemBytes, stream>>>(
            mA, mB, c, M, D, N, status, tmo);
      else
        stage_gemm_kernel<T, 64, false, true><<<grid, block, StageGemmLayout<64>::kSmemBytes, stream>>>(
            mA, mB, c, M, D, N, status, tmo);
      break;
    case Stage::kDk:  // dK[N][d] = dS[M][N]^T . Q[M][d]: both MN-major (K = M)
    case Stage::kDv:  // dV[N][d] = P[M][N]^T . dO[M][d]
      ok = encode_map(&mA, kBF16, a, N, M, H, 64) && encode_map(&mB, kBF16, b, D, M, H, 64);
      if (!ok) break;
      grid = dim3(1, (N + kTile - 1) / kTile, H);
      if (D == 128)
        stage_gemm_kernel<T, 128, true, true><<<grid, block, StageGemmLayout<128>::kSmemBytes, stream>>>(
            mA, mB, c, N, D, M, status, tmo);
      else
        stage_gemm_kernel<T, 64, true, true><<<grid, block, StageGemmLayout<64>::kSmemBytes, stream>>>(
            mA, mB, c, N, D, M, status, tmo);
      break;
  }
  if (!ok)
    return set_error(kErrInvalidArgument, "tensor map encoding failed (M=%d N=%d K_dim=%d heads=%d)", M, N, D, H);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kErrLaunch, "launch failed: %s", cudaGetErrorString(e));
  return set_error(kOk, "");
}

template <typename T>
int run_stage_softmax_bwd(const T* P, const T* dP, T* dS, int M, int N, int H) {
  if (!P || !dP || !dS) return set_error(kErrInvalidArgument, "null pointer argument");
  if (M <= 0 || N <= 0 || H <= 0)
    return set_error(kErrInvalidArgument, "sizes must be positive (M=%d N=%d heads=%d)", M, N, H);
  if (H > 65535) return set_error(kErrInvalidArgument, "total_heads=%d exceeds 65535", H);
  if (N % 8 != 0)
    return set_error(kErrMisaligned, "N=%d: [M][N] rows must be a multiple of 16 bytes (N %% 8 == 0)", N);
  if (!aligned16(P) || !aligned16(dP) || !aligned16(dS))
    return set_error(kErrMisaligned, "every buffer must be 16-byte aligned");
  if (!stage_prepare<T>()) return error_state().code.load();
  stage_softmax_bwd_kernel<T><<<dim3(M, H), kSoftmaxThreads, 0, cudaStreamLegacy>>>(P, dP, dS, M, N);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kErrLaunch, "launch failed: %s", cudaGetErrorString(e));
  return set_error(kOk, "");
}

}  // namespace fmha_sm100
