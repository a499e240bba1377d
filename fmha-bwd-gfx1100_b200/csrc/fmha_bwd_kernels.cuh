// sm_100a kernels of the attention-backward path.
//
// Reference semantics (src/kernel/correct/cpu_reference.hpp:30-40, :74-126;
// the GPU stages of src/fmha_bwd_kernels.hip:14-469):
//   dP = dO V^T,  D = rowsum(P * dP),  dS = P * (dP - D),
//   dQ = dS K,    dK = dS^T Q,          dV = P^T dO          (no scale).
//
// Two launches per call, on one stream, with no atomics anywhere:
//
//   1. dq_kernel   one CTA per (128-row query tile i, head). It walks the key
//      tiles j once. For each it computes dP_ij = dO_i V_j^T (TMEM) and, in
//      the epilogue, E_ij = P_ij * (dP_ij - c_i) in 16-bit, written back into
//      TMEM, plus the fp32 rowsum D_i += sum_n P dP. The tensor cores then
//      accumulate A_i += E_ij K_j (A operand read from TMEM) and
//      B_i += P_ij K_j. Since dS = P (dP - D) and D is only known after the
//      last key tile,
//          dQ_i = sum_j P (dP - c) K - (D - c) sum_j P K = A_i - (D_i - c_i) B_i,
//      which holds exactly for any per-row constant c_i. c_i is the
//      P-weighted mean of dP over the first key tile (an estimate of D_i), so
//      both terms stay small when dP barely varies along a row. The kernel
//      writes dQ (16-bit) and D (fp32) directly.
//
//   2. dkv_kernel  one CTA per (128-column key tile j, head). V_j stays in
//      shared memory. For every query tile i it computes dP_ij (TMEM),
//      dS_ij = P (dP - D_i) in registers (stored once to shared memory as
//      16-bit), and accumulates dV_j += P^T dO_i and dK_j += dS^T Q_i in
//      TMEM. dP and dS never reach global memory.
//
// Shared-memory tiles are loaded by TMA with 128-byte swizzle as boxes of
// 64 columns x 128 rows (16 KB). A [128][128] tile is two boxes side by side
// (box b holds columns 64b..64b+63). The same bytes serve as a K-major
// operand (K = columns) or an MN-major operand (MN = columns) depending on
// the UMMA descriptor, which is how P^T, dS^T, Q, dO and K are consumed
// without any explicit transpose.
//
// The tensor pipe accepts only about one MMA ahead of the one executing, so
// any wait (even on a barrier that has already completed) or branch in the
// issuing thread between two MMA groups idles it. dq_kernel therefore issues
// from two threads in different warps (dP in one, the two accumulations in
// the other) so that one keeps the pipe fed while the other waits; every
// hand-off between warps goes through an mbarrier (bounded waits, see
// sm100_ptx.cuh), and the streamed operands each have their own ring of
// shared-memory slots so that a slot is refilled as soon as its own last
// reader is done.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100_ptx.cuh"

namespace fmha_sm100 {

constexpr int kTile = 128;              // rows of a query tile / key tile
constexpr int kBoxCols = 64;            // columns per 128-byte swizzled box
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

// 8 consecutive keys of one row: P (one 16-byte chunk, 8 x 16-bit) times
// (dP - shift), packed back to 16-bit. Used for dS (shift = D) and for E
// (shift = c).
template <typename T>
__device__ __forceinline__ uint4 scale_chunk(uint4 pv, const uint32_t* dp, float shift) {
  const float2 ns = make_float2(-shift, -shift);
  const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 p = Elem<T>::unpack(pw[t]);
    const float2 g = make_float2(__uint_as_float(dp[2 * t]), __uint_as_float(dp[2 * t + 1]));
    const float2 r = mul_f32x2(p, add_f32x2(g, ns));
    o[t] = Elem<T>::pack(r.x, r.y);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 32 fp32 values of one row -> 64 bytes of 16-bit output.
template <typename T>
__device__ __forceinline__ void store_row_32(T* out, const float* v) {
  uint4* o = reinterpret_cast<uint4*>(out);
#pragma unroll
  for (int y = 0; y < 4; ++y) {
    o[y] = make_uint4(Elem<T>::pack(v[8 * y + 0], v[8 * y + 1]), Elem<T>::pack(v[8 * y + 2], v[8 * y + 3]),
                      Elem<T>::pack(v[8 * y + 4], v[8 * y + 5]), Elem<T>::pack(v[8 * y + 6], v[8 * y + 7]));
  }
}

// ================================================================ dq_kernel
// Shared memory: dO_i [128 x D] resident; three rings, one per streamed
// operand, so that each slot is released as soon as its own last reader is
// done: V_j (read by dP_j only), P_ij (read by B_j and by the epilogue of
// tile j) and K_j (read by B_j and A_j). D = 128: 2 slots each (224 KB);
// D = 64: 3 slots each. A 1 KB exchange area for the two warps that share
// each TMEM lane quarter (values are handed over through an mbarrier per
// quarter, so every wait is bounded); barriers.
// TMEM (512 columns): X0 [0,128), X1 [128,256) hold dP_ij; E_ij is then
// written over the first 32 columns of each 64-column half; A [256, 256+D),
// B [256+D, 256+2D).
template <int D>
struct DqCfg {
  static constexpr int kMD = (D / kBoxCols) * kBoxBytes;  // [128 x D] tile
  static constexpr int kPT = 2 * kBoxBytes;               // [128 x 128] tile
  static constexpr int kSV = D == 128 ? 2 : 3;            // V_j slots
  static constexpr int kSK = D == 128 ? 2 : 3;            // K_j slots
  static constexpr int kSP = D == 128 ? 2 : 3;            // P_ij slots
  static constexpr int kOffdO = 0;
  static constexpr int kOffV = kMD;
  static constexpr int kOffK = kOffV + kSV * kMD;
  static constexpr int kOffP = kOffK + kSK * kMD;
  static constexpr int kOffXch = kOffP + kSP * kPT;
  static constexpr int kXchBytes = 2 * kTile * 4;  // [2 halves][128 rows] fp32
  static constexpr int kOffBar = kOffXch + kXchBytes;
  static constexpr int kBarBytes = 512;
  static constexpr int kSmemBytes = kOffBar + kBarBytes + 1024;
  static constexpr int kEpiWarps = 8;
  static constexpr int kFirstEpiWarp = 2;
  static constexpr int kAbWarp = kFirstEpiWarp + kEpiWarps;  // second MMA issuer
  static constexpr int kThreads = 32 * (kAbWarp + 1);
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColX = 0;  // + 128 * buffer
  static constexpr uint32_t kColA = 256;
  static constexpr uint32_t kColB = 256 + D;
  static_assert(kColB + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum DqBar : int {
  kQbDO = 0,
  kQbVFull0 = 1,    // + slot (up to 3)
  kQbVEmpty0 = 4,   // + slot
  kQbKFull0 = 7,    // + slot
  kQbKEmpty0 = 10,  // + slot
  kQbPFull0 = 13,   // + slot
  kQbPEmpty0 = 16,  // + slot: MMA commit after B_j + 8 epilogue warps
  kQbXFull0 = 19,   // + buffer (2)
  kQbEFull0 = 21,   // + buffer
  kQbXFree0 = 23,   // + buffer
  kQbAB = 25,
  kQbDrain = 26,
  kQbXch0 = 27,     // + lane quarter (4): the two warps of a quarter swap values
  kQbDrain2 = 31,   // drain of the second MMA issuer
  kNumDqBars = 32,
};
static_assert(kNumDqBars * 8 + 8 <= 512, "dq barrier area");

template <typename T, int D>
__global__ void __launch_bounds__(DqCfg<D>::kThreads, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tm_P, const __grid_constant__ CUtensorMap tm_V,
              const __grid_constant__ CUtensorMap tm_K, const __grid_constant__ CUtensorMap tm_dO,
              T* __restrict__ dQ, float* __restrict__ Dsum, int M, int N,
              KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = DqCfg<D>;
  constexpr int SV = Cfg::kSV, SK = Cfg::kSK, SP = Cfg::kSP;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumDqBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(smem + Cfg::kOffXch);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTile;
  const int h = blockIdx.y;
  const int nt = (N + kTile - 1) / kTile;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kQbDO], 1);
    for (int s = 0; s < SV; ++s) {
      mbar_init(&bar[kQbVFull0 + s], 1);
      mbar_init(&bar[kQbVEmpty0 + s], 1);
    }
    for (int s = 0; s < SK; ++s) {
      mbar_init(&bar[kQbKFull0 + s], 1);
      mbar_init(&bar[kQbKEmpty0 + s], 1);
    }
    for (int s = 0; s < SP; ++s) {
      mbar_init(&bar[kQbPFull0 + s], 1);
      mbar_init(&bar[kQbPEmpty0 + s], 1 + Cfg::kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar[kQbXFull0 + b], 1);
      mbar_init(&bar[kQbEFull0 + b], Cfg::kEpiWarps);
      mbar_init(&bar[kQbXFree0 + b], 1);
    }
    mbar_init(&bar[kQbAB], 1);
    mbar_init(&bar[kQbDrain], 1);
    mbar_init(&bar[kQbDrain2], 1);
    for (int q = 0; q < 4; ++q) mbar_init(&bar[kQbXch0 + q], 2);
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
  WaitCtx ctx{abort_flag, timeout_ns};

  if (warp == 0) {
    // ---- TMA producer: dO_i once, then V_j, P_ij, K_j in the order the
    // tensor core needs them, each into the next slot of its own ring.
    if (lane == 0) {
      tma_prefetch_desc(&tm_P);
      tma_prefetch_desc(&tm_V);
      tma_prefetch_desc(&tm_K);
      tma_prefetch_desc(&tm_dO);
      const uint64_t pol_p = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      mbar_arrive_expect_tx(&bar[kQbDO], Cfg::kMD);
#pragma unroll
      for (int b = 0; b < D / kBoxCols; ++b)
        tma_load_3d(smem + Cfg::kOffdO + b * kBoxBytes, &tm_dO, &bar[kQbDO], b * kBoxCols, m0, h, pol_kv);
      // P streams from HBM: pull it into L2 a few key tiles ahead so the
      // shared-memory load that follows once a slot frees is an L2 hit.
      constexpr int kAhead = 4;
      auto prefetch = [&](int j) {
        tma_prefetch_l2_3d(&tm_P, j * kTile, m0, h);
        tma_prefetch_l2_3d(&tm_P, j * kTile + kBoxCols, m0, h);
      };
      for (int j = 0; j < kAhead && j < nt; ++j) prefetch(j);
      int nV = 0, nP = 0, nK = 0;  // loads issued per ring
      for (int j = 0; j < nt; ++j) {
        if (j + kAhead < nt) prefetch(j + kAhead);
        if (j >= SV && !mbar_wait(&bar[kQbVEmpty0 + j % SV], ((j / SV) - 1) & 1, ctx, 1)) break;
        {
          uint64_t* fb = &bar[kQbVFull0 + j % SV];
          uint8_t* dst = smem + Cfg::kOffV + (j % SV) * Cfg::kMD;
          mbar_arrive_expect_tx(fb, Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(dst + b * kBoxBytes, &tm_V, fb, b * kBoxCols, j * kTile, h, pol_kv);
          ++nV;
        }
        if (j >= SP && !mbar_wait(&bar[kQbPEmpty0 + j % SP], ((j / SP) - 1) & 1, ctx, 2)) break;
        {
          uint64_t* fb = &bar[kQbPFull0 + j % SP];
          uint8_t* dst = smem + Cfg::kOffP + (j % SP) * Cfg::kPT;
          mbar_arrive_expect_tx(fb, Cfg::kPT);
          tma_load_3d(dst, &tm_P, fb, j * kTile, m0, h, pol_p);
          tma_load_3d(dst + kBoxBytes, &tm_P, fb, j * kTile + kBoxCols, m0, h, pol_p);
          ++nP;
        }
        if (j >= SK && !mbar_wait(&bar[kQbKEmpty0 + j % SK], ((j / SK) - 1) & 1, ctx, 3)) break;
        {
          uint64_t* fb = &bar[kQbKFull0 + j % SK];
          uint8_t* dst = smem + Cfg::kOffK + (j % SK) * Cfg::kMD;
          mbar_arrive_expect_tx(fb, Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(dst + b * kBoxBytes, &tm_K, fb, b * kBoxCols, j * kTile, h, pol_kv);
          ++nK;
        }
      }
      if (*abort_flag) {
        // let every copy still in flight land before the CTA exits
        mbar_wait_drain(&bar[kQbDO], 0, timeout_ns);
        for (int j = (nV > SV ? nV - SV : 0); j < nV; ++j)
          mbar_wait_drain(&bar[kQbVFull0 + j % SV], (j / SV) & 1, timeout_ns);
        for (int j = (nP > SP ? nP - SP : 0); j < nP; ++j)
          mbar_wait_drain(&bar[kQbPFull0 + j % SP], (j / SP) & 1, timeout_ns);
        for (int j = (nK > SK ? nK - SK : 0); j < nK; ++j)
          mbar_wait_drain(&bar[kQbKFull0 + j % SK], (j / SK) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == Cfg::kAbWarp) {
    // ---- Two MMA issuers. The tensor pipe accepts only about one
    // instruction ahead of the one executing, so a single issuing thread
    // leaves it idle at every wait; with two, one keeps it fed while the
    // other waits. Warp 1: dP_j = dO_i V_j^T into X_(j%2). Warp kAbWarp:
    // B_j += P_ij K_j, then A_j += E_ij K_j (E from TMEM).
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      // dP = dO_i V_j^T: A = dO_i (K-major over d), B = V_j (K-major over d)
      constexpr uint32_t id_dP = make_idesc_f16<kB>(kTile, kTile, false, false);
      // A += E K_j, B += P K_j: K = keys, N = d; B operand K_j [key][d] is MN-major
      constexpr uint32_t id_AB = make_idesc_f16<kB>(kTile, D, false, true);
      const uint32_t sdO = smem_u32(smem + Cfg::kOffdO);
      const uint32_t sV0 = smem_u32(smem + Cfg::kOffV);
      const uint32_t sK0 = smem_u32(smem + Cfg::kOffK);
      const uint32_t sP0 = smem_u32(smem + Cfg::kOffP);
      bool ok = true;
      if (warp == 1) {
        ok = mbar_wait(&bar[kQbDO], 0, ctx, 13);
        for (int j = 0; j < nt && ok; ++j) {
          if (!mbar_wait(&bar[kQbVFull0 + j % SV], (j / SV) & 1, ctx, 10)) { ok = false; break; }
          if (j >= 2 && !mbar_wait(&bar[kQbXFree0 + (j & 1)], ((j >> 1) - 1) & 1, ctx, 11)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sV = sV0 + (j % SV) * Cfg::kMD;
          const uint32_t tX = tmem + Cfg::kColX + 128 * (j & 1);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
            umma_f16_ss(tX, make_sw128_desc(sdO + off, 16, 1024), make_sw128_desc(sV + off, 16, 1024), id_dP,
                        k > 0 ? 1u : 0u);
          }
          umma_commit(&bar[kQbXFull0 + (j & 1)]);
          umma_commit(&bar[kQbVEmpty0 + j % SV]);  // V_j consumed
        }
        if (!ok) {
          umma_commit(&bar[kQbDrain]);
          mbar_wait_drain(&bar[kQbDrain], 0, timeout_ns);
        }
      } else {
        for (int j = 0; j < nt && ok; ++j) {
          if (!mbar_wait(&bar[kQbPFull0 + j % SP], (j / SP) & 1, ctx, 14)) { ok = false; break; }
          if (!mbar_wait(&bar[kQbKFull0 + j % SK], (j / SK) & 1, ctx, 15)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sP = sP0 + (j % SP) * Cfg::kPT;
          const uint32_t sK = sK0 + (j % SK) * Cfg::kMD;
#pragma unroll
          for (int k = 0; k < kTile / 16; ++k) {
            umma_f16_ss(tmem + Cfg::kColB, make_sw128_desc(sP + (k >> 2) * kBoxBytes + (k & 3) * 32, 16, 1024),
                        make_sw128_desc(sK + k * 2048, kBoxBytes, 1024), id_AB, (j > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&bar[kQbPEmpty0 + j % SP]);  // the tensor core's read of P_ij
          if (!mbar_wait(&bar[kQbEFull0 + (j & 1)], (j >> 1) & 1, ctx, 12)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tE = tmem + Cfg::kColX + 128 * (j & 1);
#pragma unroll
          for (int k = 0; k < kTile / 16; ++k) {
            // E for keys 16k..16k+15 sits in key half (k >> 2): 8 columns per step
            umma_f16_ts(tmem + Cfg::kColA, tE + (k >> 2) * 64 + (k & 3) * 8,
                        make_sw128_desc(sK + k * 2048, kBoxBytes, 1024), id_AB, (j > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&bar[kQbKEmpty0 + j % SK]);  // K_j consumed (B_j and A_j)
          umma_commit(&bar[kQbXFree0 + (j & 1)]);
        }
        if (ok) {
          umma_commit(&bar[kQbAB]);
        } else {
          umma_commit(&bar[kQbDrain2]);
          mbar_wait_drain(&bar[kQbDrain2], 0, timeout_ns);
        }
      }
    }
  } else {
    // ---- Epilogue: 8 warps. Warp w owns TMEM lane quarter q = w % 4 (query
    // rows 32q..32q+31 of the tile) and key half c (keys 64c..64c+63 of each
    // key tile). The two warps of a quarter swap per-row values through xch,
    // synchronised by mbarrier kQbXch0 + q (both warps arrive once per round).
    const int q = warp & 3;
    const int c = (warp - Cfg::kFirstEpiWarp) >> 2;
    const int r = q * 32 + lane;
    const int m = m0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t rsw = static_cast<uint32_t>(r);
    float Dacc = 0.f;   // this half's sum_n P dP over all key tiles
    float shift = 0.f;  // c_i
    uint32_t xphase = 0;
    // One round: both warps of the quarter have arrived.
    auto xch_round = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kQbXch0 + q]);
      const bool w = mbar_wait(&bar[kQbXch0 + q], xphase & 1, ctx, 23);
      ++xphase;
      __syncwarp();
      return w;
    };
    // Partner's value for this row; `reuse` adds the round that lets the
    // partner read before xch is written again.
    auto swap = [&](float mine, float& other, bool reuse) -> bool {
      xch[c * kTile + r] = mine;
      if (!xch_round()) return false;
      other = xch[(1 - c) * kTile + r];
      return reuse ? xch_round() : true;
    };
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      const int s = j % SP;
      const int b = j & 1;
      if (!mbar_wait(&bar[kQbXFull0 + b], (j >> 1) & 1, ctx, 20)) { ok = false; break; }
      if (!mbar_wait(&bar[kQbPFull0 + s], (j / SP) & 1, ctx, 21)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      uint32_t dpa[32], dpb[32];
      tmem_load_32(lane_base + Cfg::kColX + 128 * b + 64 * c, dpa);
      tmem_load_32(lane_base + Cfg::kColX + 128 * b + 64 * c + 32, dpb);
      const uint8_t* pbox = smem + Cfg::kOffP + s * Cfg::kPT + c * kBoxBytes;
      uint4 pv[8];
#pragma unroll
      for (int x = 0; x < 8; ++x) pv[x] = *reinterpret_cast<const uint4*>(pbox + sw128_offset(rsw, x));
      // sum_n P dP (and, on the first key tile, sum_n P for the shift)
      float sp = 0.f, spdp = 0.f;
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const uint32_t pw[4] = {pv[x].x, pv[x].y, pv[x].z, pv[x].w};
        const uint32_t* dp = x < 4 ? dpa + 8 * x : dpb + 8 * (x - 4);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float2 p = Elem<T>::unpack(pw[t]);
          spdp = fmaf(p.x, __uint_as_float(dp[2 * t]), spdp);
          spdp = fmaf(p.y, __uint_as_float(dp[2 * t + 1]), spdp);
          sp += p.x + p.y;
        }
      }
      Dacc += spdp;
      if (j == 0) {
        // shift c_i = P-weighted mean of dP over key tile 0 (both halves)
        float sp_o = 0.f, spdp_o = 0.f;
        if (!swap(sp, sp_o, true) || !swap(spdp, spdp_o, true)) { ok = false; break; }
        const float sp_all = sp + sp_o;
        shift = sp_all > 1e-30f ? (spdp + spdp_o) / sp_all : 0.f;
      }
      // E = P (dP - c) in 16-bit, 32 packed columns at X_b + 64c
      uint32_t e[32];
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const uint4 ev = scale_chunk<T>(pv[x], x < 4 ? dpa + 8 * x : dpb + 8 * (x - 4), shift);
        e[4 * x + 0] = ev.x;
        e[4 * x + 1] = ev.y;
        e[4 * x + 2] = ev.z;
        e[4 * x + 3] = ev.w;
      }
      tmem_store_32(lane_base + Cfg::kColX + 128 * b + 64 * c, e);
      tmem_store_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[kQbEFull0 + b]);
        mbar_arrive(&bar[kQbPEmpty0 + s]);
      }
    }
    // dQ = A - (D - c) B, and D
    if (ok && mbar_wait(&bar[kQbAB], 0, ctx, 22)) {
      __syncwarp();
      tc_fence_after();
      float Dother = 0.f;
      const bool swapped = swap(Dacc, Dother, false);
      const float Dfull = Dacc + Dother;
      const float sD = Dfull - shift;
      constexpr int kHalf = D / 2;
      T* out = dQ + (static_cast<int64_t>(h) * M + m) * D + c * kHalf;
#pragma unroll
      for (int x = 0; x < kHalf / 32; ++x) {
        uint32_t a[32], bb[32];
        tmem_load_32(lane_base + Cfg::kColA + c * kHalf + 32 * x, a);
        tmem_load_32(lane_base + Cfg::kColB + c * kHalf + 32 * x, bb);
        float v[32];
#pragma unroll
        for (int y = 0; y < 32; ++y) v[y] = fmaf(-sD, __uint_as_float(bb[y]), __uint_as_float(a[y]));
        if (swapped && m < M) store_row_32<T>(out + 32 * x, v);
      }
      if (swapped && c == 0 && m < M) Dsum[static_cast<int64_t>(h) * M + m] = Dfull;
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) publish_failure(*abort_flag, status);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// =============================================================== dkv_kernel
// Shared memory (D = 128): V_j 32 KB, P_ij x2 64 KB, dS 32 KB, dO_i x2 64 KB,
// Q_i 32 KB = 224 KB. TMEM: two dP buffers [0,256) (lane = query row, column
// = key), dV [256,256+D) and dK [256+D,256+2D) (lane = key row, column = d).
//
// Warp roles (12 warps): 0 TMA for V_j and the P stream; 1 MMA issuer for
// dP (and TMEM owner); 2 TMA for dO_i and Q_i; 3 MMA issuer for dV and dK;
// 4-11 dS warps (TMEM lane quarter = warp % 4, key half = (warp - 4) / 4),
// which also write dK_j, dV_j.
template <int D>
struct DkvCfg {
  static constexpr int kMD = (D / kBoxCols) * kBoxBytes;
  static constexpr int kPT = 2 * kBoxBytes;
  static constexpr int kOffV = 0;
  static constexpr int kOffP = kOffV + kMD;  // two stages
  static constexpr int kOffS = kOffP + 2 * kPT;
  static constexpr int kOffdO = kOffS + kPT;  // two stages
  static constexpr int kOffQ = kOffdO + 2 * kMD;
  static constexpr int kTileBytes = kOffQ + kMD;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kTileBytes + kBarBytes + 1024;
  static constexpr int kDSWarps = 8;
  static constexpr int kFirstDSWarp = 4;
  static constexpr int kThreads = 32 * (kFirstDSWarp + kDSWarps);
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColdP = 0;  // + 128 * buffer (two dP buffers)
  static constexpr uint32_t kColdV = 256;
  static constexpr uint32_t kColdK = 256 + D;
  static_assert(kColdK + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum DkvBar : int {
  kKbV = 0,
  kKbPFull0 = 1,
  kKbPEmpty0 = 3,
  kKbDOFull0 = 5,
  kKbDOEmpty0 = 7,
  kKbQFull = 9,
  kKbQEmpty = 10,
  kKbDPFull0 = 11,   // + dP buffer (2)
  kKbDPEmpty0 = 13,  // + dP buffer
  kKbDSFull = 15,
  kKbDSEmpty = 16,
  kKbAcc = 17,
  kKbDrain = 18,
  kKbDrain2 = 19,
  kNumDkvBars = 20,
};

template <typename T, int D>
__global__ void __launch_bounds__(DkvCfg<D>::kThreads, 1)
    dkv_kernel(const __grid_constant__ CUtensorMap tm_Q, const __grid_constant__ CUtensorMap tm_V,
               const __grid_constant__ CUtensorMap tm_dO, const __grid_constant__ CUtensorMap tm_P,
               const float* __restrict__ Dsum, T* __restrict__ dK, T* __restrict__ dV, int M, int N,
               KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = DkvCfg<D>;
  constexpr int kEpi = Cfg::kDSWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumDkvBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTile;
  const int h = blockIdx.y;
  const int mt = (M + kTile - 1) / kTile;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kKbV], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[kKbPFull0 + s], 1);
      mbar_init(&bar[kKbPEmpty0 + s], 1 + kEpi);
      mbar_init(&bar[kKbDOFull0 + s], 1);
      mbar_init(&bar[kKbDOEmpty0 + s], 2);  // read by dP_i and dV_i (two issuers)
    }
    mbar_init(&bar[kKbQFull], 1);
    mbar_init(&bar[kKbQEmpty], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar[kKbDPFull0 + b], 1);
      mbar_init(&bar[kKbDPEmpty0 + b], kEpi);
    }
    mbar_init(&bar[kKbDSFull], kEpi);
    mbar_init(&bar[kKbDSEmpty], 1);
    mbar_init(&bar[kKbAcc], 1);
    mbar_init(&bar[kKbDrain], 1);
    mbar_init(&bar[kKbDrain2], 1);
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
  WaitCtx ctx{abort_flag, timeout_ns};

  if (warp == 0) {
    // ---- TMA producer: V_j once, then the P stream (2 stages).
    if (lane == 0) {
      tma_prefetch_desc(&tm_V);
      tma_prefetch_desc(&tm_P);
      const uint64_t pol_p = l2_policy_evict_first();
      const uint64_t pol_v = l2_policy_evict_normal();
      mbar_arrive_expect_tx(&bar[kKbV], Cfg::kMD);
#pragma unroll
      for (int b = 0; b < D / kBoxCols; ++b)
        tma_load_3d(smem + Cfg::kOffV + b * kBoxBytes, &tm_V, &bar[kKbV], b * kBoxCols, n0, h, pol_v);
      constexpr int kAhead = 4;  // P tiles pulled into L2 ahead of the 2-stage ring
      for (int i = 0; i < kAhead && i < mt; ++i) {
        tma_prefetch_l2_3d(&tm_P, n0, i * kTile, h);
        tma_prefetch_l2_3d(&tm_P, n0 + kBoxCols, i * kTile, h);
      }
      int issued = 0;
      for (int i = 0; i < mt; ++i) {
        const int s = i & 1;
        const int u = i >> 1;
        if (i + kAhead < mt) {
          tma_prefetch_l2_3d(&tm_P, n0, (i + kAhead) * kTile, h);
          tma_prefetch_l2_3d(&tm_P, n0 + kBoxCols, (i + kAhead) * kTile, h);
        }
        if (u > 0 && !mbar_wait(&bar[kKbPEmpty0 + s], (u - 1) & 1, ctx, 30)) break;
        uint8_t* dst = smem + Cfg::kOffP + s * Cfg::kPT;
        mbar_arrive_expect_tx(&bar[kKbPFull0 + s], Cfg::kPT);
        tma_load_3d(dst, &tm_P, &bar[kKbPFull0 + s], n0, i * kTile, h, pol_p);
        tma_load_3d(dst + kBoxBytes, &tm_P, &bar[kKbPFull0 + s], n0 + kBoxCols, i * kTile, h, pol_p);
        ++issued;
      }
      if (*abort_flag) {
        mbar_wait_drain(&bar[kKbV], 0, timeout_ns);
        for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i)
          mbar_wait_drain(&bar[kKbPFull0 + (i & 1)], (i >> 1) & 1, timeout_ns);
      }
    }
  } else if (warp == 2) {
    // ---- TMA producer for the L2-resident operands: dO_i (2 slots) and Q_i
    // (1 slot). Polls both "empty" barriers without blocking and issues
    // whichever load can go; tiles are prefetched into L2 kL2Ahead query
    // tiles ahead (every key-tile CTA of the head reads them).
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
        if (next_do < mt) {
          const int s = next_do & 1;
          const int u = next_do >> 1;
          if (u == 0 || mbar_poll(&bar[kKbDOEmpty0 + s], (u - 1) & 1)) {
            mbar_arrive_expect_tx(&bar[kKbDOFull0 + s], Cfg::kMD);
#pragma unroll
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_load_3d(smem + Cfg::kOffdO + s * Cfg::kMD + b * kBoxBytes, &tm_dO, &bar[kKbDOFull0 + s],
                          b * kBoxCols, next_do * kTile, h, pol);
            if (next_do + kL2Ahead < mt)
              for (int b = 0; b < D / kBoxCols; ++b)
                tma_prefetch_l2_3d(&tm_dO, b * kBoxCols, (next_do + kL2Ahead) * kTile, h);
            ++next_do;
            progressed = true;
          }
        }
        if (next_q < mt && (next_q == 0 || mbar_poll(&bar[kKbQEmpty], (next_q - 1) & 1))) {
          mbar_arrive_expect_tx(&bar[kKbQFull], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffQ + b * kBoxBytes, &tm_Q, &bar[kKbQFull], b * kBoxCols,
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
            note_failure(ctx, 31);
            failed = true;
          }
        }
      }
      if (*abort_flag) {
        for (int i = (next_do > 2 ? next_do - 2 : 0); i < next_do; ++i)
          mbar_wait_drain(&bar[kKbDOFull0 + (i & 1)], (i >> 1) & 1, timeout_ns);
        if (next_q > 0) mbar_wait_drain(&bar[kKbQFull], (next_q - 1) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == 3) {
    // ---- Two MMA issuers (one keeps the tensor pipe fed while the other
    // waits). Warp 1: dP_i = dO_i V_j^T. Warp 3: dV_j += P_ij^T dO_i and
    // dK_j += dS_ij^T Q_i in the order dV_0 dV_1 dK_0 dV_2 dK_1 ..., so the
    // dS epilogue of tile i overlaps dV_{i+1}.
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      constexpr uint32_t id_dP = make_idesc_f16<kB>(kTile, kTile, false, false);
      constexpr uint32_t id_dVK = make_idesc_f16<kB>(kTile, D, true, true);
      const uint32_t sV = smem_u32(smem + Cfg::kOffV);
      const uint32_t sS = smem_u32(smem + Cfg::kOffS);
      const uint32_t sQ = smem_u32(smem + Cfg::kOffQ);
      bool ok = true;
      if (warp == 1) {
        ok = mbar_wait(&bar[kKbV], 0, ctx, 45);
        for (int i = 0; i < mt && ok; ++i) {
          const int s = i & 1;
          const uint32_t sdO = smem_u32(smem + Cfg::kOffdO + s * Cfg::kMD);
          // dP = dO_i V_j^T : A = dO_i (K-major over d), B = V_j (K-major over d).
          if (!mbar_wait(&bar[kKbDOFull0 + s], (i >> 1) & 1, ctx, 40)) { ok = false; break; }
          // dP buffer b = i % 2 is free once the dS warps have read dP_{i-2}
          if (i >= 2 && !mbar_wait(&bar[kKbDPEmpty0 + (i & 1)], ((i >> 1) - 1) & 1, ctx, 41)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
            umma_f16_ss(tmem + Cfg::kColdP + 128 * (i & 1), make_sw128_desc(sdO + off, 16, 1024),
                        make_sw128_desc(sV + off, 16, 1024), id_dP, k > 0 ? 1u : 0u);
          }
          umma_commit(&bar[kKbDPFull0 + (i & 1)]);
          umma_commit(&bar[kKbDOEmpty0 + s]);
        }
        if (!ok) {
          umma_commit(&bar[kKbDrain]);
          mbar_wait_drain(&bar[kKbDrain], 0, timeout_ns);
        }
      } else {
        auto issue_dV = [&](int i) -> bool {
          const int s = i & 1;
          const uint32_t sdO = smem_u32(smem + Cfg::kOffdO + s * Cfg::kMD);
          const uint32_t sP = smem_u32(smem + Cfg::kOffP + s * Cfg::kPT);
          // dV += P_ij^T dO_i : A = P^T (MN-major, M = key), B = dO_i (MN-major, N = d).
          if (!mbar_wait(&bar[kKbPFull0 + s], (i >> 1) & 1, ctx, 42)) return false;
          if (!mbar_wait(&bar[kKbDOFull0 + s], (i >> 1) & 1, ctx, 46)) return false;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < kTile / 16; ++k) {
            umma_f16_ss(tmem + Cfg::kColdV, make_sw128_desc(sP + k * 2048, kBoxBytes, 1024),
                        make_sw128_desc(sdO + k * 2048, kBoxBytes, 1024), id_dVK, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&bar[kKbDOEmpty0 + s]);
          umma_commit(&bar[kKbPEmpty0 + s]);
          return true;
        };
        auto issue_dK = [&](int i) -> bool {
          // dK += dS^T Q_i : A = dS^T (MN-major, M = key), B = Q_i (MN-major, N = d).
          if (!mbar_wait(&bar[kKbQFull], i & 1, ctx, 43)) return false;
          if (!mbar_wait(&bar[kKbDSFull], i & 1, ctx, 44)) return false;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < kTile / 16; ++k) {
            umma_f16_ss(tmem + Cfg::kColdK, make_sw128_desc(sS + k * 2048, kBoxBytes, 1024),
                        make_sw128_desc(sQ + k * 2048, kBoxBytes, 1024), id_dVK, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&bar[kKbQEmpty]);
          umma_commit(&bar[kKbDSEmpty]);
          return true;
        };
        ok = issue_dV(0);
        for (int i = 0; i < mt && ok; ++i) {
          if (i + 1 < mt && !issue_dV(i + 1)) { ok = false; break; }
          if (!issue_dK(i)) { ok = false; break; }
        }
        if (ok) {
          umma_commit(&bar[kKbAcc]);
        } else {
          umma_commit(&bar[kKbDrain2]);
          mbar_wait_drain(&bar[kKbDrain2], 0, timeout_ns);
        }
      }
    }
  } else if (warp >= Cfg::kFirstDSWarp) {
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
      const int b = i & 1;
      if (!mbar_wait(&bar[kKbDPFull0 + b], (i >> 1) & 1, ctx, 50)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      // Both 32-column halves of this warp's dP segment are loaded before any
      // other work, then the TMEM buffer is released.
      uint32_t dpa[32], dpb[32];
      tmem_load_32(lane_base + Cfg::kColdP + 128 * b + c * 64, dpa);
      tmem_load_32(lane_base + Cfg::kColdP + 128 * b + c * 64 + 32, dpb);
      if (!mbar_wait(&bar[kKbPFull0 + s], (i >> 1) & 1, ctx, 51)) { ok = false; break; }
      __syncwarp();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kKbDPEmpty0 + b]);
      const uint8_t* pbox = smem + Cfg::kOffP + s * Cfg::kPT + c * kBoxBytes;
      uint4 ds[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 pv = *reinterpret_cast<const uint4*>(pbox + sw128_offset(rsw, j));
        ds[j] = scale_chunk<T>(pv, dpa + 8 * j, Dm);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 pv = *reinterpret_cast<const uint4*>(pbox + sw128_offset(rsw, 4 + j));
        ds[4 + j] = scale_chunk<T>(pv, dpb + 8 * j, Dm);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kKbPEmpty0 + s]);
      if (i > 0 && !mbar_wait(&bar[kKbDSEmpty], (i - 1) & 1, ctx, 52)) { ok = false; break; }
      __syncwarp();
      uint8_t* sbox = smem + Cfg::kOffS + c * kBoxBytes;
#pragma unroll
      for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(sbox + sw128_offset(rsw, j)) = ds[j];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kKbDSFull]);
    }
    // final dV_j and dK_j rows (lane = key row) -> 16-bit outputs
    if (ok && mbar_wait(&bar[kKbAcc], 0, ctx, 53)) {
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
          if (n < N) store_row_32<T>(out + x * 32, reinterpret_cast<const float*>(v));
        }
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) publish_failure(*abort_flag, status);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace fmha_sm100
