// sm_100a kernels of the attention-backward path.
//
// Reference semantics (src/kernel/correct/cpu_reference.hpp:30-40, :74-126;
// the GPU stages of src/fmha_bwd_kernels.hip:14-469):
//   dP = dO V^T,  D = rowsum(P * dP),  dS = P * (dP - D),
//   dQ = dS K,    dK = dS^T Q,          dV = P^T dO          (no scale).
//
// Three launches per call, all on one stream:
//   1. rowsum_kernel   one CTA per (128-row query tile, head). Computes
//                      O = P V on the tensor cores (TMEM accumulator) and
//                      D[m] = sum_k dO[m,k] O[m,k], which equals
//                      sum_n P[m,n] dP[m,n]. Also zeroes the fp32 dQ
//                      accumulator rows of its tile.
//   2. main_kernel     one CTA per (128-column key tile, head). K_j and V_j
//                      stay in shared memory; for every 128-row query tile i
//                      it computes dP = dO_i V_j^T (TMEM), dS in registers
//                      (written once to shared memory as 16-bit), and
//                      accumulates dV_j += P^T dO_i and dK_j += dS^T Q_i in
//                      TMEM; dQ_i partial = dS K_j goes through TMEM into the
//                      fp32 accumulator with vector reductions. dP and dS
//                      never reach global memory.
//   3. dq_finalize     converts the fp32 dQ accumulator to the 16-bit output.
//
// Shared-memory tiles are loaded by TMA with 128-byte swizzle as boxes of
// 64 columns x 128 rows (16 KB). A [128][128] tile is two boxes side by side
// (box b holds columns 64b..64b+63). The same bytes serve as a K-major
// operand (K = columns) or an MN-major operand (MN = columns) depending on
// the UMMA descriptor, which is how P^T, dS^T, Q, dO and K are consumed
// without any explicit transpose.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100_ptx.cuh"

namespace fmha_sm100 {

constexpr int kTile = 128;          // rows of a query tile / key tile
constexpr int kBoxCols = 64;        // columns per 128-byte swizzled box
constexpr int kBoxBytes = kTile * 128;  // 16 KB

// ------------------------------------------------------------ type traits
template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
  static constexpr bool kBF16 = true;
  __device__ __forceinline__ static float2 unpack(uint32_t v) {
    float2 r;
    r.x = __uint_as_float(v << 16);
    r.y = __uint_as_float(v & 0xFFFF0000u);
    return r;
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <>
struct Elem<__half> {
  static constexpr bool kBF16 = false;
  __device__ __forceinline__ static float2 unpack(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled box (the TMA SWIZZLE_128B pattern: chunk ^= row % 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ------------------------------------------------------------- rowsum
// Shared-memory plan: kStages x { P tile [128 x 128] (32 KB), V tile
// [128 x D] (D/64 boxes) }.
template <int D>
struct RowsumCfg {
  static constexpr int kPBytes = 2 * kBoxBytes;
  static constexpr int kVBytes = (D / kBoxCols) * kBoxBytes;
  static constexpr int kStageBytes = kPBytes + kVBytes;
  static constexpr int kStages = D == 128 ? 3 : 4;
  static constexpr int kTileBytes = kStages * kStageBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kTileBytes + kBarBytes + 1024;  // +1024: alignment slack
  static constexpr int kThreads = 192;  // warp0 TMA, warp1 MMA, warps 2-5 epilogue
  static constexpr uint32_t kTmemCols = D;  // O accumulator [128 x D] fp32
};

template <typename T, int D>
__global__ void __launch_bounds__(RowsumCfg<D>::kThreads, 1)
    rowsum_kernel(const __grid_constant__ CUtensorMap tm_P,
                  const __grid_constant__ CUtensorMap tm_V, const T* __restrict__ dO,
                  float* __restrict__ Dsum, float* __restrict__ dQacc, int M, int N,
                  KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = RowsumCfg<D>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kTileBytes);
  uint64_t* full = bars;            // [S]
  uint64_t* empty = bars + S;       // [S]
  uint64_t* o_full = bars + 2 * S;  // [1]
  uint64_t* drain = bars + 2 * S + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTile;
  const int h = blockIdx.y;
  const int nt = (N + kTile - 1) / kTile;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  WaitCtx ctx{abort_flag, status, timeout_ns};

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_P);
      tma_prefetch_desc(&tm_V);
      const uint64_t pol_p = l2_policy_evict_normal();
      const uint64_t pol_v = l2_policy_evict_last();
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nt && ok; ++j) {
        const int s = j % S;
        const int u = j / S;
        if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1, ctx, 1)) { ok = false; break; }
        uint8_t* st = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
        tma_load_3d(st, &tm_P, &full[s], j * kTile, m0, h, pol_p);
        tma_load_3d(st + kBoxBytes, &tm_P, &full[s], j * kTile + kBoxCols, m0, h, pol_p);
#pragma unroll
        for (int b = 0; b < D / kBoxCols; ++b)
          tma_load_3d(st + Cfg::kPBytes + b * kBoxBytes, &tm_V, &full[s], b * kBoxCols,
                      j * kTile, h, pol_v);
        ++issued;
      }
      if (!ok) {
        // Let every load this thread issued land before the CTA exits.
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
          mbar_wait_drain(&full[j % S], (j / S) & 1, timeout_ns);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16<Elem<T>::kBF16>(kTile, D, false, true);
      bool ok = true;
      for (int j = 0; j < nt; ++j) {
        const int s = j % S;
        const int u = j / S;
        if (!mbar_wait(&full[s], u & 1, ctx, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + s * Cfg::kStageBytes);
        const uint32_t v_addr = p_addr + Cfg::kPBytes;
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          // A = P tile, K-major over the key index n (16 keys per step).
          const uint64_t a = make_sw128_desc(p_addr + (k >> 2) * kBoxBytes + (k & 3) * 32, 16, 1024);
          // B = V tile [n][d], MN-major (N = d), K = n: 16 rows per step.
          const uint64_t b = make_sw128_desc(v_addr + k * 2048, kBoxBytes, 1024);
          umma_f16_ss(tmem, a, b, idesc, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) {
        umma_commit(o_full);
      } else {
        umma_commit(drain);
        mbar_wait_drain(drain, 0, timeout_ns);
      }
    }
  } else {
    // Epilogue: warps 2..5 -> TMEM lane quarter (warp % 4), one row each.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int m = m0 + r;
    const bool ok = mbar_wait(o_full, 0, ctx, 3);
    __syncwarp();  // lanes leave the wait loop independently; tcgen05.ld is .aligned
    if (ok) {
      tc_fence_after();
      float acc = 0.f;
      const T* dO_row = dO + (static_cast<int64_t>(h) * M + m) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_load_32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c * 32, v);
        if (m < M) {
          const uint4* src = reinterpret_cast<const uint4*>(dO_row + c * 32);
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            const uint4 w = __ldg(src + x);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              const float2 f = Elem<T>::unpack(ww[y]);
              acc = fmaf(f.x, __uint_as_float(v[x * 8 + y * 2]), acc);
              acc = fmaf(f.y, __uint_as_float(v[x * 8 + y * 2 + 1]), acc);
            }
          }
        }
      }
      tc_fence_before();
      if (m < M) {
        Dsum[static_cast<int64_t>(h) * M + m] = acc;
        float4* z = reinterpret_cast<float4*>(dQacc + (static_cast<int64_t>(h) * M + m) * D);
#pragma unroll
        for (int x = 0; x < D / 4; ++x) z[x] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// --------------------------------------------------------------- main
// Shared-memory plan (D = 128): K_j 32 KB, V_j 32 KB, P_ij x2 64 KB, dS 32 KB,
// dO_i 32 KB, Q_i 32 KB = 224 KB.
// TMEM (512 columns): dP [0,128) (lane = query row, column = key),
// dV [128,128+D) and dK [128+D,128+2D) (lane = key row, column = d), and the
// dQ partial at [128+2D, ...):
//   D = 128: dQ^T = K_j^T dS^T, lane = d, column = query row (128 columns),
//            so each warp reduces 32 consecutive floats of one dQ row per
//            instruction (one 128-byte line);
//   D = 64:  dQ = dS K_j, lane = query row, column = d (64 columns).
//
// Warp roles (20 warps): 0 TMA for K_j, V_j and the P stream; 1 MMA issuer
// for dP and dV (and TMEM owner); 2 TMA for dO_i and Q_i; 3 MMA issuer for
// dK and dQ; 4-11 dS warps (TMEM lane
// quarter = warp % 4, column half = (warp - 4) / 4), which also write the
// final dK_j, dV_j; 12-19 dQ warps (lane quarter = warp % 4, column half =
// (warp - 12) / 4). A dQ warp first copies its 64 TMEM columns of the dQ
// partial into registers and releases the TMEM, then issues the global
// reductions, so the reduction traffic never holds up the next dQ MMA.
template <int D>
struct MainCfg {
  static constexpr int kMD = (D / kBoxCols) * kBoxBytes;  // one [128 x D] tile
  static constexpr int kPT = 2 * kBoxBytes;               // one [128 x 128] tile
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kOffK + kMD;
  static constexpr int kOffP = kOffV + kMD;  // two stages
  static constexpr int kOffS = kOffP + 2 * kPT;
  static constexpr int kOffdO = kOffS + kPT;
  static constexpr int kOffQ = kOffdO + kMD;
  static constexpr int kTileBytes = kOffQ + kMD;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kTileBytes + kBarBytes + 1024;
  static constexpr int kDSWarps = 8;
  static constexpr int kDQWarps = 8;
  static constexpr int kFirstDSWarp = 4;
  static constexpr int kFirstDQWarp = kFirstDSWarp + kDSWarps;
  static constexpr int kThreads = 32 * (kFirstDQWarp + kDQWarps);
  static constexpr bool kDQTransposed = (D == 128);
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColdP = 0;
  static constexpr uint32_t kColdV = 128;
  static constexpr uint32_t kColdK = 128 + D;
  static constexpr uint32_t kColdQ = 128 + 2 * D;
  static constexpr uint32_t kdQCols = kDQTransposed ? kTile : D;
  static_assert(kColdQ + kdQCols <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Barrier indices inside the main kernel's barrier block.
enum MainBar : int {
  kBarKV = 0,
  kBarPFull0 = 1,
  kBarPFull1 = 2,
  kBarPEmpty0 = 3,
  kBarPEmpty1 = 4,
  kBarDOFull = 5,
  kBarDOEmpty = 6,
  kBarQFull = 7,
  kBarQEmpty = 8,
  kBarDPFull = 9,
  kBarDPEmpty = 10,
  kBarDSFull = 11,
  kBarDSEmpty = 12,
  kBarDQFull = 13,
  kBarDQEmpty = 14,
  kBarAccFull = 15,
  kBarDrain = 16,
  kBarDrain2 = 17,
  kNumMainBars = 18,
};

// dS for 8 consecutive keys of one row: P (8 x 16-bit, one 16-byte chunk)
// times (dP - D), packed back to 16-bit.
template <typename T>
__device__ __forceinline__ uint4 ds_chunk(uint4 pv, const uint32_t* dp, float Dm) {
  const float2 nD = make_float2(-Dm, -Dm);
  const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 p = Elem<T>::unpack(pw[t]);
    const float2 g = make_float2(__uint_as_float(dp[2 * t]), __uint_as_float(dp[2 * t + 1]));
    const float2 r = mul_f32x2(p, add_f32x2(g, nD));
    o[t] = Elem<T>::pack(r.x, r.y);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <typename T, int D>
__global__ void __launch_bounds__(MainCfg<D>::kThreads, 1)
    main_kernel(const __grid_constant__ CUtensorMap tm_Q,
                const __grid_constant__ CUtensorMap tm_K,
                const __grid_constant__ CUtensorMap tm_V,
                const __grid_constant__ CUtensorMap tm_dO,
                const __grid_constant__ CUtensorMap tm_P, const float* __restrict__ Dsum,
                float* __restrict__ dQacc, T* __restrict__ dK, T* __restrict__ dV, int M,
                int N, KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = MainCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumMainBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTile;
  const int h = blockIdx.y;
  const int mt = (M + kTile - 1) / kTile;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kBarKV], 1);
    mbar_init(&bar[kBarPFull0], 1);
    mbar_init(&bar[kBarPFull1], 1);
    mbar_init(&bar[kBarPEmpty0], 1 + Cfg::kDSWarps);
    mbar_init(&bar[kBarPEmpty1], 1 + Cfg::kDSWarps);
    mbar_init(&bar[kBarDOFull], 1);
    mbar_init(&bar[kBarDOEmpty], 1);
    mbar_init(&bar[kBarQFull], 1);
    mbar_init(&bar[kBarQEmpty], 1);
    mbar_init(&bar[kBarDPFull], 1);
    mbar_init(&bar[kBarDPEmpty], Cfg::kDSWarps);
    mbar_init(&bar[kBarDSFull], Cfg::kDSWarps);
    mbar_init(&bar[kBarDSEmpty], 1);
    mbar_init(&bar[kBarDQFull], 1);
    mbar_init(&bar[kBarDQEmpty], Cfg::kDQWarps);
    mbar_init(&bar[kBarAccFull], 2);
    mbar_init(&bar[kBarDrain], 1);
    mbar_init(&bar[kBarDrain2], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  WaitCtx ctx{abort_flag, status, timeout_ns};

  if (warp == 0) {
    // ---- TMA producer: K_j, V_j once, then the P stream (2 stages).
    if (lane == 0) {
      tma_prefetch_desc(&tm_K);
      tma_prefetch_desc(&tm_V);
      tma_prefetch_desc(&tm_P);
      const uint64_t pol_kv = l2_policy_evict_normal();
      const uint64_t pol_p = l2_policy_evict_first();
      mbar_arrive_expect_tx(&bar[kBarKV], 2 * Cfg::kMD);
#pragma unroll
      for (int b = 0; b < D / kBoxCols; ++b) {
        tma_load_3d(smem + Cfg::kOffK + b * kBoxBytes, &tm_K, &bar[kBarKV], b * kBoxCols, n0, h, pol_kv);
        tma_load_3d(smem + Cfg::kOffV + b * kBoxBytes, &tm_V, &bar[kBarKV], b * kBoxCols, n0, h, pol_kv);
      }
      int issued = 0;
      for (int i = 0; i < mt; ++i) {
        const int s = i & 1;
        const int u = i >> 1;
        if (u > 0 && !mbar_wait(&bar[kBarPEmpty0 + s], (u - 1) & 1, ctx, 10)) break;
        uint8_t* dst = smem + Cfg::kOffP + s * Cfg::kPT;
        mbar_arrive_expect_tx(&bar[kBarPFull0 + s], Cfg::kPT);
        tma_load_3d(dst, &tm_P, &bar[kBarPFull0 + s], n0, i * kTile, h, pol_p);
        tma_load_3d(dst + kBoxBytes, &tm_P, &bar[kBarPFull0 + s], n0 + kBoxCols, i * kTile, h, pol_p);
        ++issued;
      }
      if (*abort_flag) {
        mbar_wait_drain(&bar[kBarKV], 0, timeout_ns);
        for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i)
          mbar_wait_drain(&bar[kBarPFull0 + (i & 1)], (i >> 1) & 1, timeout_ns);
      }
    }
  } else if (warp == 2) {
    // ---- TMA producer for the L2-resident operands dO_i and Q_i
    // (single-buffered each). It polls both "empty" barriers without
    // blocking and issues whichever load can go, so neither stream waits
    // behind the other. Tiles are first prefetched into L2 kL2Ahead query
    // tiles ahead (they are shared by every key-tile CTA of the head).
    if (lane == 0) {
      constexpr int kL2Ahead = 3;
      tma_prefetch_desc(&tm_dO);
      tma_prefetch_desc(&tm_Q);
      const uint64_t pol = l2_policy_evict_last();
      for (int i = 0; i < kL2Ahead && i < mt; ++i)
        for (int b = 0; b < D / kBoxCols; ++b) {
          tma_prefetch_l2_3d(&tm_dO, b * kBoxCols, i * kTile, h);
          tma_prefetch_l2_3d(&tm_Q, b * kBoxCols, i * kTile, h);
        }
      int next_do = 0, next_q = 0;
      uint64_t t_last = global_timer_ns();
      bool failed = false;
      while ((next_do < mt || next_q < mt) && !failed) {
        bool progressed = false;
        if (next_do < mt && (next_do == 0 || mbar_test(&bar[kBarDOEmpty], (next_do - 1) & 1))) {
          mbar_arrive_expect_tx(&bar[kBarDOFull], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffdO + b * kBoxBytes, &tm_dO, &bar[kBarDOFull], b * kBoxCols,
                        next_do * kTile, h, pol);
          if (next_do + kL2Ahead < mt)
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_prefetch_l2_3d(&tm_dO, b * kBoxCols, (next_do + kL2Ahead) * kTile, h);
          ++next_do;
          progressed = true;
        }
        if (next_q < mt && (next_q == 0 || mbar_test(&bar[kBarQEmpty], (next_q - 1) & 1))) {
          mbar_arrive_expect_tx(&bar[kBarQFull], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffQ + b * kBoxBytes, &tm_Q, &bar[kBarQFull], b * kBoxCols,
                        next_q * kTile, h, pol);
          if (next_q + kL2Ahead < mt)
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_prefetch_l2_3d(&tm_Q, b * kBoxCols, (next_q + kL2Ahead) * kTile, h);
          ++next_q;
          progressed = true;
        }
        if (progressed) {
          t_last = global_timer_ns();
        } else {
          if (*abort_flag) break;
          if (global_timer_ns() - t_last > timeout_ns) {
            record_failure(ctx, kStatusWaitTimeout, 20);
            failed = true;
          }
        }
      }
      if (*abort_flag) {
        if (next_do > 0) mbar_wait_drain(&bar[kBarDOFull], (next_do - 1) & 1, timeout_ns);
        if (next_q > 0) mbar_wait_drain(&bar[kBarQFull], (next_q - 1) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == 3) {
    // ---- MMA issuers: warp 1 issues dP and dV, warp 3 issues dK and dQ.
    // Two issuing threads keep the tensor pipe fed while either one waits.
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      constexpr uint32_t id_dP = make_idesc_f16<kB>(kTile, kTile, false, false);
      constexpr uint32_t id_dVK = make_idesc_f16<kB>(kTile, D, true, true);
      // D = 128: dQ^T (M = d, N = query rows; A = K_j^T MN-major, B = dS^T K-major).
      // D = 64:  dQ   (M = query rows, N = d; A = dS K-major, B = K_j MN-major).
      constexpr uint32_t id_dQ = Cfg::kDQTransposed ? make_idesc_f16<kB>(kTile, kTile, true, false)
                                                    : make_idesc_f16<kB>(kTile, D, false, true);
      const uint32_t sK = smem_u32(smem + Cfg::kOffK);
      const uint32_t sV = smem_u32(smem + Cfg::kOffV);
      const uint32_t sS = smem_u32(smem + Cfg::kOffS);
      const uint32_t sdO = smem_u32(smem + Cfg::kOffdO);
      const uint32_t sQ = smem_u32(smem + Cfg::kOffQ);
      const uint32_t t_dP = tmem + Cfg::kColdP;
      const uint32_t t_dV = tmem + Cfg::kColdV;
      const uint32_t t_dK = tmem + Cfg::kColdK;
      const uint32_t t_dQ = tmem + Cfg::kColdQ;
      // Issue order is software-pipelined by one query tile:
      //   dP_0 dV_0 | dP_1 dV_1 dK_0 dQ_0 | dP_2 dV_2 dK_1 dQ_1 | ...
      // so the dS epilogue of tile i overlaps dK_{i-1}, dQ_{i-1}, dP_{i+1}
      // and dV_{i+1} on the tensor pipe.
      auto issue_dP_dV = [&](int i) -> bool {
        const int s = i & 1;
        const uint32_t sP = smem_u32(smem + Cfg::kOffP + s * Cfg::kPT);
        // dP = dO_i V_j^T : A = dO_i (K-major over d), B = V_j (K-major over d).
        if (!mbar_wait(&bar[kBarDOFull], i & 1, ctx, 31)) return false;
        if (i > 0 && !mbar_wait(&bar[kBarDPEmpty], (i - 1) & 1, ctx, 32)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
          umma_f16_ss(t_dP, make_sw128_desc(sdO + off, 16, 1024),
                      make_sw128_desc(sV + off, 16, 1024), id_dP, k > 0 ? 1u : 0u);
        }
        umma_commit(&bar[kBarDPFull]);
        // dV += P_ij^T dO_i : A = P^T (MN-major, M = key), B = dO_i (MN-major, N = d).
        if (!mbar_wait(&bar[kBarPFull0 + s], (i >> 1) & 1, ctx, 33)) return false;
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          umma_f16_ss(t_dV, make_sw128_desc(sP + k * 2048, kBoxBytes, 1024),
                      make_sw128_desc(sdO + k * 2048, kBoxBytes, 1024), id_dVK,
                      (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&bar[kBarDOEmpty]);
        umma_commit(&bar[kBarPEmpty0 + s]);
        return true;
      };
      auto issue_dK_dQ = [&](int i) -> bool {
        // dK += dS^T Q_i : A = dS^T (MN-major, M = key), B = Q_i (MN-major, N = d).
        if (!mbar_wait(&bar[kBarQFull], i & 1, ctx, 34)) return false;
        if (!mbar_wait(&bar[kBarDSFull], i & 1, ctx, 35)) return false;
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          umma_f16_ss(t_dK, make_sw128_desc(sS + k * 2048, kBoxBytes, 1024),
                      make_sw128_desc(sQ + k * 2048, kBoxBytes, 1024), id_dVK,
                      (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&bar[kBarQEmpty]);
        // dQ partial over this key tile (reduction over the 128 keys).
        if (i > 0 && !mbar_wait(&bar[kBarDQEmpty], (i - 1) & 1, ctx, 36)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          const uint64_t ds_kmajor =
              make_sw128_desc(sS + (k >> 2) * kBoxBytes + (k & 3) * 32, 16, 1024);
          const uint64_t k_mnmajor = make_sw128_desc(sK + k * 2048, kBoxBytes, 1024);
          if constexpr (Cfg::kDQTransposed)
            umma_f16_ss(t_dQ, k_mnmajor, ds_kmajor, id_dQ, k > 0 ? 1u : 0u);
          else
            umma_f16_ss(t_dQ, ds_kmajor, k_mnmajor, id_dQ, k > 0 ? 1u : 0u);
        }
        umma_commit(&bar[kBarDQFull]);
        umma_commit(&bar[kBarDSEmpty]);
        return true;
      };
      const bool is_a = (warp == 1);
      bool ok = mbar_wait(&bar[kBarKV], 0, ctx, 30);
      for (int i = 0; i < mt && ok; ++i) ok = is_a ? issue_dP_dV(i) : issue_dK_dQ(i);
      uint64_t* drain = &bar[is_a ? kBarDrain : kBarDrain2];
      if (ok) {
        umma_commit(&bar[kBarAccFull]);
      } else {
        umma_commit(drain);
        mbar_wait_drain(drain, 0, timeout_ns);
      }
    }
  } else if (warp >= Cfg::kFirstDSWarp && warp < Cfg::kFirstDQWarp) {
    // ---- dS warps.
    const int q = warp & 3;
    const int c = (warp - Cfg::kFirstDSWarp) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t rsw = static_cast<uint32_t>(r);
    bool ok = true;
    for (int i = 0; i < mt && ok; ++i) {
      const int s = i & 1;
      const int m = i * kTile + r;
      const float Dm = (m < M) ? __ldg(Dsum + static_cast<int64_t>(h) * M + m) : 0.f;
      if (!mbar_wait(&bar[kBarDPFull], i & 1, ctx, 40)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      // Both 32-column halves of this warp's dP segment are loaded before any
      // other work, then the TMEM is released.
      uint32_t dpa[32], dpb[32];
      tmem_load_32(lane_base + Cfg::kColdP + c * 64, dpa);
      tmem_load_32(lane_base + Cfg::kColdP + c * 64 + 32, dpb);
      if (!mbar_wait(&bar[kBarPFull0 + s], (i >> 1) & 1, ctx, 41)) { ok = false; break; }
      __syncwarp();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kBarDPEmpty]);
      const uint8_t* pbox = smem + Cfg::kOffP + s * Cfg::kPT + c * kBoxBytes;
      uint4 ds[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 pv = *reinterpret_cast<const uint4*>(pbox + sw128_offset(rsw, j));
        ds[j] = ds_chunk<T>(pv, dpa + 8 * j, Dm);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 pv = *reinterpret_cast<const uint4*>(pbox + sw128_offset(rsw, 4 + j));
        ds[4 + j] = ds_chunk<T>(pv, dpb + 8 * j, Dm);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kBarPEmpty0 + s]);
      if (i > 0 && !mbar_wait(&bar[kBarDSEmpty], (i - 1) & 1, ctx, 42)) { ok = false; break; }
      uint8_t* sbox = smem + Cfg::kOffS + c * kBoxBytes;
#pragma unroll
      for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(sbox + sw128_offset(rsw, j)) = ds[j];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kBarDSFull]);
    }
    // final dV_j and dK_j rows (lane = key row) -> 16-bit outputs
    if (ok && mbar_wait(&bar[kBarAccFull], 0, ctx, 44)) {
      __syncwarp();
      tc_fence_after();
      const int n = n0 + r;
      constexpr int kHalf = D / 2;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = (which == 0 ? Cfg::kColdV : Cfg::kColdK) + c * kHalf;
        T* out = (which == 0 ? dV : dK) + (static_cast<int64_t>(h) * N + n) * D + c * kHalf;
#pragma unroll
        for (int x = 0; x < kHalf / 32; ++x) {
          uint32_t v[32];
          tmem_load_32(lane_base + col + x * 32, v);
          if (n < N) {
            uint4* o = reinterpret_cast<uint4*>(out + x * 32);
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              o[y] = make_uint4(Elem<T>::pack(__uint_as_float(v[8 * y + 0]), __uint_as_float(v[8 * y + 1])),
                                Elem<T>::pack(__uint_as_float(v[8 * y + 2]), __uint_as_float(v[8 * y + 3])),
                                Elem<T>::pack(__uint_as_float(v[8 * y + 4]), __uint_as_float(v[8 * y + 5])),
                                Elem<T>::pack(__uint_as_float(v[8 * y + 6]), __uint_as_float(v[8 * y + 7])));
            }
          }
        }
      }
      tc_fence_before();
    }
  } else if (warp >= Cfg::kFirstDQWarp) {
    // ---- dQ warps: TMEM -> registers -> fp32 accumulator.
    const int q = warp & 3;
    const int c = (warp - Cfg::kFirstDQWarp) >> 2;
    constexpr int kCols = Cfg::kdQCols / 2;  // columns of the dQ partial per warp
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + Cfg::kColdQ + c * kCols;
    for (int i = 0; i < mt; ++i) {
      if (!mbar_wait(&bar[kBarDQFull], i & 1, ctx, 50)) break;
      __syncwarp();
      tc_fence_after();
      uint32_t v[kCols];
      if constexpr (kCols == 64)
        tmem_load_64(lane_base, *reinterpret_cast<uint32_t(*)[64]>(&v[0]));
      else
        tmem_load_32(lane_base, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kBarDQEmpty]);
      const int mbase = i * kTile;
      if constexpr (Cfg::kDQTransposed) {
        // lane = d (32q + lane), column = query row mbase + c*64 + j: one
        // 128-byte line of a dQ row per warp-wide reduction.
        const int m0 = mbase + c * kCols;
        const int valid = min(kCols, M - m0);
        float* p = dQacc + (static_cast<int64_t>(h) * M + m0) * D + q * 32 + lane;
#pragma unroll
        for (int j = 0; j < kCols; ++j)
          if (j < valid) red_add_f32(p + static_cast<int64_t>(j) * D, __uint_as_float(v[j]));
      } else {
        // lane = query row (32q + lane), column = d (c*32 .. c*32+31).
        const int m = mbase + q * 32 + lane;
        if (m < M) {
          float* dst = dQacc + (static_cast<int64_t>(h) * M + m) * D + c * kCols;
#pragma unroll
          for (int y = 0; y < kCols / 4; ++y)
            red_add_v4_f32(dst + 4 * y, __uint_as_float(v[4 * y]), __uint_as_float(v[4 * y + 1]),
                           __uint_as_float(v[4 * y + 2]), __uint_as_float(v[4 * y + 3]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------ finalize
// dQ = T(dQacc), 8 elements per thread per iteration. Block 0 also copies the
// call's status word to the host-visible slot and clears it for the next call.
template <typename T>
__global__ void __launch_bounds__(256)
    dq_finalize_kernel(const float* __restrict__ dQacc, T* __restrict__ dQ, int64_t count,
                       KernelStatus* status, KernelStatus* host_status) {
  const int64_t n8 = count / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(dQacc) + 2 * i);
    const float4 b = __ldcs(reinterpret_cast<const float4*>(dQacc) + 2 * i + 1);
    reinterpret_cast<uint4*>(dQ)[i] = make_uint4(Elem<T>::pack(a.x, a.y), Elem<T>::pack(a.z, a.w),
                                                 Elem<T>::pack(b.x, b.y), Elem<T>::pack(b.z, b.w));
  }
  // tail (count not a multiple of 8)
  for (int64_t i = n8 * 8 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += stride) {
    const float v = dQacc[i];
    const uint32_t p = Elem<T>::pack(v, 0.f);
    reinterpret_cast<uint16_t*>(dQ)[i] = static_cast<uint16_t>(p & 0xFFFFu);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && host_status != nullptr) {
    volatile KernelStatus* hs = host_status;
    hs->code = status->code;
    hs->where = status->where;
    hs->block = status->block;
    status->code = 0;
    status->where = 0;
    status->block = 0;
  }
}

}  // namespace fmha_sm100
