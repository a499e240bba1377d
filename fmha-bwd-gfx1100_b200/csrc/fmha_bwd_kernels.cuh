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
//      shared memory. For every query tile i it computes dP_ij^T (TMEM, key
//      index on the lanes), dS_ij^T = P^T (dP^T - D_i) in registers, written
//      back into TMEM as 16-bit, and accumulates dV_j += P^T dO_i and
//      dK_j += dS^T Q_i (A operand from TMEM) in TMEM. dP and dS never reach
//      global memory.
//
// Both kernels are persistent (one CTA per SM walking the work items).
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

// Coalesced store of 16-bit output rows held one row per lane: lane l has
// the S 16-byte chunks (8 values each) of row l, at byte offset 16 j of the
// row for chunk j. An S x S transpose of the chunks within each group of S
// lanes (log2 S butterfly stages of __shfl_xor_sync; stage m swaps bit m of
// the lane and chunk indices) leaves lane l with chunk l % S of rows
// S (l / S) + k, k = 0..S-1, so that each of the S stores writes 32 / S
// whole 16 S-byte row segments instead of 32 scattered 16-byte pieces.
// Rows at or past `valid` are not written. All 32 lanes must call this.
template <int S>
__device__ __forceinline__ void store_rows_coalesced(uint4 (&c)[S], uint8_t* row0, size_t pitch,
                                                     int lane, int valid) {
#pragma unroll
  for (int m = 1; m < S; m <<= 1) {
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int j = 0; j < S; ++j) {
      if (j & m) continue;
      const uint4 snd = hi ? c[j] : c[j ^ m];
      uint4 rcv;
      rcv.x = __shfl_xor_sync(0xffffffffu, snd.x, m);
      rcv.y = __shfl_xor_sync(0xffffffffu, snd.y, m);
      rcv.z = __shfl_xor_sync(0xffffffffu, snd.z, m);
      rcv.w = __shfl_xor_sync(0xffffffffu, snd.w, m);
      if (hi) c[j] = rcv;
      else c[j ^ m] = rcv;
    }
  }
  const int g0 = lane & ~(S - 1), i = lane & (S - 1);
#pragma unroll
  for (int k = 0; k < S; ++k) {
    const int row = g0 + k;
    if (row < valid) *reinterpret_cast<uint4*>(row0 + static_cast<size_t>(row) * pitch + 16 * i) = c[k];
  }
}

// Work units of the persistent kernels. Items are walked by the CTAs in
// waves of gridDim.x; when the last wave would be less than half full, its
// items (the tail) are split into `parts` parts each, so they fill one wave:
// units [0, full) are whole items, units [full, full + parts * tail) are the
// parts of items full.. (part p covers steps [p len / parts, (p + 1) len /
// parts) of the item's len steps). A part leaves fp32 partial results in a
// workspace slot (unit - full); a combine kernel, launched after the main
// kernel on the same stream, adds them up and writes the item's outputs.
constexpr int kMaxParts = 4;  // parts per split item, at most
struct UnitMap {
  int full;   // whole items
  int parts;  // parts per tail item (1: no split)
  int units;  // full + parts * (items - full)
  __device__ __forceinline__ void get(int u, int len, int& item, int& lo, int& hi, int& part) const {
    if (u < full) {
      item = u;
      lo = 0;
      hi = len;
      part = -1;
      return;
    }
    const int v = u - full;
    const int k = v / parts;
    item = full + k;
    part = v - k * parts;
    lo = (part * len) / parts;
    hi = ((part + 1) * len) / parts;
  }
};

// ================================================================ dq_kernel
// Shared memory: dO_i [128 x D] resident; three rings, one per streamed
// operand, so that each slot is released as soon as its own last reader is
// done: V_j (read by dP_j only), P_ij (read by B_j and by the epilogue of
// tile j) and K_j (read by B_j and A_j). D = 128: 2 slots each (224 KB);
// D = 64: 3 slots each. A 1 KB exchange area for the two warps that share
// each TMEM lane quarter (values are handed over through an mbarrier per
// quarter, so every wait is bounded); barriers.
// TMEM (512 columns): buffers X_b [128 b, 128 b + 128) hold dP_ij (two at
// D = 128, three at D = 64); E_ij is then written over the first 32 columns
// of each 64-column half; A and B (D columns each) follow.
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
  // D = 64: B and A have an issuing thread each (kBWarp, kAWarp); D = 128:
  // kBWarp issues both (at D = 128 the split measured slower).
  static constexpr bool kSplit = D == 64;
  static constexpr int kBWarp = kFirstEpiWarp + kEpiWarps;  // MMA issuer of B (and A)
  static constexpr int kAWarp = kBWarp + 1;                   // MMA issuer of A (D = 64)
  static constexpr int kThreads = 32 * (kBWarp + 1 + (kSplit ? 1 : 0));
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kNX = D == 128 ? 2 : 3;  // dP/E buffers
  static constexpr uint32_t kColX = 0;          // + 128 * buffer
  static constexpr uint32_t kColA = 128 * kNX;
  static constexpr uint32_t kColB = kColA + D;
  static_assert(kColB + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum DqBar : int {
  kQbDO = 0,
  kQbVFull0 = 1,    // + slot (up to 3)
  kQbVEmpty0 = 4,   // + slot
  kQbKFull0 = 7,    // + slot
  kQbKEmpty0 = 10,  // + slot: commits of B_j and A_j
  kQbPFull0 = 13,   // + slot
  kQbPEmpty0 = 16,  // + slot: MMA commit after B_j + 8 epilogue warps
  kQbXFull0 = 19,   // + buffer (up to 3)
  kQbEFull0 = 22,   // + buffer
  kQbXFree0 = 25,   // + buffer
  kQbAB = 28,       // A and B of an item complete (a commit from each issuer)
  kQbDrain = 29,
  kQbXch0 = 30,     // + lane quarter (4): the two warps of a quarter swap values
  kQbDrain2 = 34,   // drain of the second MMA issuer
  kQbDOEmpty = 35,  // the dP MMAs of an item are done with dO_i
  kQbAccEmpty = 36, // the dS warps have read an item's A and B (8 warps)
  kQbDrain3 = 37,   // drain of the third MMA issuer
  kNumDqBars = 38,
};
static_assert(kNumDqBars * 8 + 8 <= 512, "dq barrier area");

// kGivenD: D (rowsum of P * dP, one float per query row and head) is an
// input; then E = P (dP - D) = dS, A = dS K = dQ directly, and neither the
// B accumulation nor the rowsum is needed (5 instead of 6 GEMM-sized MMA
// passes per call). Otherwise Dsum is written.
template <typename T, int D, bool kGivenD = false>
__global__ void __launch_bounds__(DqCfg<D>::kThreads, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tm_P, const __grid_constant__ CUtensorMap tm_V,
              const __grid_constant__ CUtensorMap tm_K, const __grid_constant__ CUtensorMap tm_dO,
              T* __restrict__ dQ, float* __restrict__ Dsum, int M, int N, int H, UnitMap um,
              float* __restrict__ part_ws, KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = DqCfg<D>;
  constexpr int SV = Cfg::kSV, SK = Cfg::kSK, SP = Cfg::kSP, NX = Cfg::kNX;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumDqBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(smem + Cfg::kOffXch);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt = (M + kTile - 1) / kTile;
  const int nt = (N + kTile - 1) / kTile;
  // work items (query tile, head), head-major, walked as work units (um): a
  // unit is an item's key tiles [lo, hi)

  if (threadIdx.x == 0) {
    mbar_init(&bar[kQbDO], 1);
    mbar_init(&bar[kQbDOEmpty], 1);
    for (int s = 0; s < SV; ++s) {
      mbar_init(&bar[kQbVFull0 + s], 1);
      mbar_init(&bar[kQbVEmpty0 + s], 1);
    }
    for (int s = 0; s < SK; ++s) {
      mbar_init(&bar[kQbKFull0 + s], 1);
      mbar_init(&bar[kQbKEmpty0 + s], (Cfg::kSplit && !kGivenD) ? 2 : 1);
    }
    for (int s = 0; s < SP; ++s) {
      mbar_init(&bar[kQbPFull0 + s], 1);
      mbar_init(&bar[kQbPEmpty0 + s], 1 + Cfg::kEpiWarps);
    }
    for (int b = 0; b < Cfg::kNX; ++b) {
      mbar_init(&bar[kQbXFull0 + b], 1);
      mbar_init(&bar[kQbEFull0 + b], Cfg::kEpiWarps);
      mbar_init(&bar[kQbXFree0 + b], 1);
    }
    mbar_init(&bar[kQbAB], (Cfg::kSplit && !kGivenD) ? 2 : 1);
    mbar_init(&bar[kQbAccEmpty], Cfg::kEpiWarps);
    mbar_init(&bar[kQbDrain], 1);
    mbar_init(&bar[kQbDrain2], 1);
    mbar_init(&bar[kQbDrain3], 1);
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

  // Every role walks the same work units: u = blockIdx.x, + gridDim.x, ...
  // Shared-memory rings, TMEM buffers and their barrier phases continue
  // across units (global step counter g over (unit, key tile)).
  if (warp == 0) {
    // ---- TMA producer: per item dO_i (once the previous item's dP MMAs are
    // done), then V_j, P_ij, K_j in the order the tensor core needs them.
    if (lane == 0) {
      tma_prefetch_desc(&tm_P);
      tma_prefetch_desc(&tm_V);
      tma_prefetch_desc(&tm_K);
      tma_prefetch_desc(&tm_dO);
      const uint64_t pol_p = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      // No L2 prefetch ahead of the rings: prefetch requests share the TMA
      // unit and L2 queues with the loads, and with them every kernel took
      // 3-7 % more SM cycles.
      int g = 0, nV = 0, nP = 0, nK = 0, nD = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x) {
        int t, lo, hi, part;
        um.get(u, nt, t, lo, hi, part);
        const int h = t / mt;
        const int m0 = (t - h * mt) * kTile;
        if (nD > 0 && !mbar_wait(&bar[kQbDOEmpty], (nD - 1) & 1, ctx, 4)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar[kQbDO], Cfg::kMD);
#pragma unroll
        for (int b = 0; b < D / kBoxCols; ++b)
          tma_load_3d(smem + Cfg::kOffdO + b * kBoxBytes, &tm_dO, &bar[kQbDO], b * kBoxCols, m0, h, pol_kv);
        ++nD;
        for (int j = lo; j < hi; ++j, ++g) {
          if (g >= SV && !mbar_wait(&bar[kQbVEmpty0 + g % SV], ((g / SV) - 1) & 1, ctx, 1)) { ok = false; break; }
          {
            uint64_t* fb = &bar[kQbVFull0 + g % SV];
            uint8_t* dst = smem + Cfg::kOffV + (g % SV) * Cfg::kMD;
            mbar_arrive_expect_tx(fb, Cfg::kMD);
#pragma unroll
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_load_3d(dst + b * kBoxBytes, &tm_V, fb, b * kBoxCols, j * kTile, h, pol_kv);
            ++nV;
          }
          if (g >= SP && !mbar_wait(&bar[kQbPEmpty0 + g % SP], ((g / SP) - 1) & 1, ctx, 2)) { ok = false; break; }
          {
            uint64_t* fb = &bar[kQbPFull0 + g % SP];
            uint8_t* dst = smem + Cfg::kOffP + (g % SP) * Cfg::kPT;
            mbar_arrive_expect_tx(fb, Cfg::kPT);
            tma_load_3d(dst, &tm_P, fb, j * kTile, m0, h, pol_p);
            tma_load_3d(dst + kBoxBytes, &tm_P, fb, j * kTile + kBoxCols, m0, h, pol_p);
            ++nP;
          }
          if (g >= SK && !mbar_wait(&bar[kQbKEmpty0 + g % SK], ((g / SK) - 1) & 1, ctx, 3)) { ok = false; break; }
          {
            uint64_t* fb = &bar[kQbKFull0 + g % SK];
            uint8_t* dst = smem + Cfg::kOffK + (g % SK) * Cfg::kMD;
            mbar_arrive_expect_tx(fb, Cfg::kMD);
#pragma unroll
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_load_3d(dst + b * kBoxBytes, &tm_K, fb, b * kBoxCols, j * kTile, h, pol_kv);
            ++nK;
          }
        }
      }
      if (*abort_flag) {
        // let every copy still in flight land before the CTA exits
        if (nD > 0) mbar_wait_drain(&bar[kQbDO], (nD - 1) & 1, timeout_ns);
        for (int j = (nV > SV ? nV - SV : 0); j < nV; ++j)
          mbar_wait_drain(&bar[kQbVFull0 + j % SV], (j / SV) & 1, timeout_ns);
        for (int j = (nP > SP ? nP - SP : 0); j < nP; ++j)
          mbar_wait_drain(&bar[kQbPFull0 + j % SP], (j / SP) & 1, timeout_ns);
        for (int j = (nK > SK ? nK - SK : 0); j < nK; ++j)
          mbar_wait_drain(&bar[kQbKFull0 + j % SK], (j / SK) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == Cfg::kBWarp || warp == Cfg::kAWarp) {
    // ---- MMA issuers. The tensor pipe accepts only about one instruction
    // ahead of the one executing, and a thread between two of its MMA groups
    // spends a few hundred cycles on barrier waits and commits, so the work
    // is spread over several issuing threads that keep the pipe fed while one
    // waits. Warp 1: dP_j = dO_i V_j^T into X_(g%2). Warp kBWarp:
    // B_j += P_ij K_j, and at D = 128 then A_j += E_ij K_j (E from TMEM); at
    // D = 64 warp kAWarp issues A_j. B and A start an item once the epilogue
    // has read the previous item's A and B.
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      // dP = dO_i V_j^T: A = dO_i (K-major over d), B = V_j (K-major over d)
      constexpr uint32_t id_dP = make_idesc_f16<kB>(kTile, kTile, false, false);
      // A += E K_j, B += P K_j: K = keys, N = d; B operand K_j [key][d] is MN-major
      constexpr uint32_t id_AB = make_idesc_f16<kB>(kTile, D, false, true);
      const uint64_t ddO = make_sw128_desc(smem_u32(smem + Cfg::kOffdO), 16, 1024);
      const uint32_t sV0 = smem_u32(smem + Cfg::kOffV);
      const uint32_t sK0 = smem_u32(smem + Cfg::kOffK);
      const uint32_t sP0 = smem_u32(smem + Cfg::kOffP);
      bool ok = true;
      int g = 0, tc = 0;
      if (warp == 1) {
        for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
          int t, lo, hi, part;
          um.get(u, nt, t, lo, hi, part);
          if (!mbar_wait(&bar[kQbDO], tc & 1, ctx, 13)) { ok = false; break; }
          for (int j = lo; j < hi; ++j, ++g) {
            if (!mbar_wait(&bar[kQbVFull0 + g % SV], (g / SV) & 1, ctx, 10)) { ok = false; break; }
            if (g >= NX && !mbar_wait(&bar[kQbXFree0 + g % NX], ((g / NX) - 1) & 1, ctx, 11)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dV = make_sw128_desc(sV0 + (g % SV) * Cfg::kMD, 16, 1024);
            const uint32_t tX = tmem + Cfg::kColX + 128 * (g % NX);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
              umma_f16_ss(tX, desc_advance(ddO, off), desc_advance(dV, off), id_dP, k > 0 ? 1u : 0u);
            }
            umma_commit(&bar[kQbXFull0 + g % NX]);
            umma_commit(&bar[kQbVEmpty0 + g % SV]);  // V_j consumed
          }
          if (ok) umma_commit(&bar[kQbDOEmpty]);  // dO_i consumed
        }
        if (!ok) {
          umma_commit(&bar[kQbDrain]);
          mbar_wait_drain(&bar[kQbDrain], 0, timeout_ns);
        }
      } else if (warp == Cfg::kBWarp && !Cfg::kSplit) {
        for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
          int t, lo, hi, part;
          um.get(u, nt, t, lo, hi, part);
          if (tc > 0 && !mbar_wait(&bar[kQbAccEmpty], (tc - 1) & 1, ctx, 16)) { ok = false; break; }
          for (int j = lo; j < hi; ++j, ++g) {
            if (!kGivenD && !mbar_wait(&bar[kQbPFull0 + g % SP], (g / SP) & 1, ctx, 14)) { ok = false; break; }
            if (!mbar_wait(&bar[kQbKFull0 + g % SK], (g / SK) & 1, ctx, 15)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dK = make_sw128_desc(sK0 + (g % SK) * Cfg::kMD, kBoxBytes, 1024);
            if constexpr (!kGivenD) {
              const uint64_t dP = make_sw128_desc(sP0 + (g % SP) * Cfg::kPT, 16, 1024);
#pragma unroll
              for (int k = 0; k < kTile / 16; ++k) {
                umma_f16_ss(tmem + Cfg::kColB, desc_advance(dP, (k >> 2) * kBoxBytes + (k & 3) * 32),
                            desc_advance(dK, k * 2048), id_AB, (j > lo || k > 0) ? 1u : 0u);
              }
              umma_commit(&bar[kQbPEmpty0 + g % SP]);  // the tensor core's read of P_ij
            }
            if (!mbar_wait(&bar[kQbEFull0 + g % NX], (g / NX) & 1, ctx, 12)) { ok = false; break; }
            tc_fence_after();
            const uint32_t tE = tmem + Cfg::kColX + 128 * (g % NX);
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              // E for keys 16k..16k+15 sits in key half (k >> 2): 8 columns per step
              umma_f16_ts(tmem + Cfg::kColA, tE + (k >> 2) * 64 + (k & 3) * 8, desc_advance(dK, k * 2048), id_AB,
                          (j > lo || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[kQbKEmpty0 + g % SK]);  // K_j consumed (B_j and A_j)
            umma_commit(&bar[kQbXFree0 + g % NX]);
            if (kGivenD) umma_commit(&bar[kQbPEmpty0 + g % SP]);  // keeps the slot's arrival count
          }
          if (ok) umma_commit(&bar[kQbAB]);  // A and B of this item complete
        }
        if (!ok) {
          umma_commit(&bar[kQbDrain2]);
          mbar_wait_drain(&bar[kQbDrain2], 0, timeout_ns);
        }
      } else if (warp == Cfg::kBWarp) {
        if constexpr (!kGivenD) {
          for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
            int t, lo, hi, part;
            um.get(u, nt, t, lo, hi, part);
            if (tc > 0 && !mbar_wait(&bar[kQbAccEmpty], (tc - 1) & 1, ctx, 16)) { ok = false; break; }
            for (int j = lo; j < hi; ++j, ++g) {
              if (!mbar_wait(&bar[kQbPFull0 + g % SP], (g / SP) & 1, ctx, 14)) { ok = false; break; }
              if (!mbar_wait(&bar[kQbKFull0 + g % SK], (g / SK) & 1, ctx, 15)) { ok = false; break; }
              tc_fence_after();
              const uint64_t dK = make_sw128_desc(sK0 + (g % SK) * Cfg::kMD, kBoxBytes, 1024);
              const uint64_t dP = make_sw128_desc(sP0 + (g % SP) * Cfg::kPT, 16, 1024);
#pragma unroll
              for (int k = 0; k < kTile / 16; ++k) {
                umma_f16_ss(tmem + Cfg::kColB, desc_advance(dP, (k >> 2) * kBoxBytes + (k & 3) * 32),
                            desc_advance(dK, k * 2048), id_AB, (j > lo || k > 0) ? 1u : 0u);
              }
              umma_commit(&bar[kQbPEmpty0 + g % SP]);  // the tensor core's read of P_ij
              umma_commit(&bar[kQbKEmpty0 + g % SK]);
            }
            if (ok) umma_commit(&bar[kQbAB]);
          }
          if (!ok) {
            umma_commit(&bar[kQbDrain2]);
            mbar_wait_drain(&bar[kQbDrain2], 0, timeout_ns);
          }
        }
      } else {
        for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
          int t, lo, hi, part;
          um.get(u, nt, t, lo, hi, part);
          if (tc > 0 && !mbar_wait(&bar[kQbAccEmpty], (tc - 1) & 1, ctx, 19)) { ok = false; break; }
          for (int j = lo; j < hi; ++j, ++g) {
            if (!mbar_wait(&bar[kQbKFull0 + g % SK], (g / SK) & 1, ctx, 18)) { ok = false; break; }
            if (!mbar_wait(&bar[kQbEFull0 + g % NX], (g / NX) & 1, ctx, 12)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dK = make_sw128_desc(sK0 + (g % SK) * Cfg::kMD, kBoxBytes, 1024);
            const uint32_t tE = tmem + Cfg::kColX + 128 * (g % NX);
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              // E for keys 16k..16k+15 sits in key half (k >> 2): 8 columns per step
              umma_f16_ts(tmem + Cfg::kColA, tE + (k >> 2) * 64 + (k & 3) * 8, desc_advance(dK, k * 2048), id_AB,
                          (j > lo || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[kQbKEmpty0 + g % SK]);  // K_j consumed (B_j and A_j)
            umma_commit(&bar[kQbXFree0 + g % NX]);
            if (kGivenD) umma_commit(&bar[kQbPEmpty0 + g % SP]);  // keeps the slot's arrival count
          }
          if (ok) umma_commit(&bar[kQbAB]);  // A (and, from kBWarp, B) of this item complete
        }
        if (!ok) {
          umma_commit(&bar[kQbDrain3]);
          mbar_wait_drain(&bar[kQbDrain3], 0, timeout_ns);
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
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t rsw = static_cast<uint32_t>(r);
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
    // Partner's value for this row; the second round lets the partner read
    // before xch is written again.
    auto swap = [&](float mine, float& other) -> bool {
      xch[c * kTile + r] = mine;
      if (!xch_round()) return false;
      other = xch[(1 - c) * kTile + r];
      return xch_round();
    };
    bool ok = true;
    int g = 0, tc = 0;
    for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
      int t, lo, hi, part;
      um.get(u, nt, t, lo, hi, part);
      const int h = t / mt;
      const int m = (t - h * mt) * kTile + r;
      float Dacc = 0.f;   // this half's sum_n P dP over the unit's key tiles
      float shift = 0.f;  // c (D_i itself when D is given)
      if constexpr (kGivenD) shift = m < M ? Dsum[static_cast<int64_t>(h) * M + m] : 0.f;
      for (int j = lo; j < hi; ++j, ++g) {
        const int s = g % SP;
        const int b = g % NX;  // dP/E buffer
        if (!mbar_wait(&bar[kQbXFull0 + b], (g / NX) & 1, ctx, 20)) { ok = false; break; }
        if (!mbar_wait(&bar[kQbPFull0 + s], (g / SP) & 1, ctx, 21)) { ok = false; break; }
        __syncwarp();
        tc_fence_after();
        uint32_t dpa[32], dpb[32];
        tmem_load_32(lane_base + Cfg::kColX + 128 * b + 64 * c, dpa);
        tmem_load_32(lane_base + Cfg::kColX + 128 * b + 64 * c + 32, dpb);
        const uint8_t* pbox = smem + Cfg::kOffP + s * Cfg::kPT + c * kBoxBytes;
        uint4 pv[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) pv[x] = *reinterpret_cast<const uint4*>(pbox + sw128_offset(rsw, x));
        // sum_n P dP over this half tile
        float spdp = 0.f;
        if constexpr (!kGivenD) {
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            const uint32_t pw[4] = {pv[x].x, pv[x].y, pv[x].z, pv[x].w};
            const uint32_t* dp = x < 4 ? dpa + 8 * x : dpb + 8 * (x - 4);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 p = Elem<T>::unpack(pw[u]);
              spdp = fmaf(p.x, __uint_as_float(dp[2 * u]), spdp);
              spdp = fmaf(p.y, __uint_as_float(dp[2 * u + 1]), spdp);
            }
          }
          Dacc += spdp;
        }
        if (!kGivenD && j == lo) {
          // shift c = P-weighted mean of dP over the unit's first key tile
          // (both halves)
          float sp = 0.f;
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            const uint32_t pw[4] = {pv[x].x, pv[x].y, pv[x].z, pv[x].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 p = Elem<T>::unpack(pw[u]);
              sp += p.x + p.y;
            }
          }
          float sp_o = 0.f, spdp_o = 0.f;
          if (!swap(sp, sp_o) || !swap(spdp, spdp_o)) { ok = false; break; }
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
      if (!ok) break;
      // dQ = A - (D - c) B, and D (or dQ = A when D is given); then hand A
      // and B back to the issuer. A part of a split item leaves its A, B,
      // partial D and shift c in the workspace instead, and dq_combine_kernel
      // adds them up: dQ = sum_p (A_p - (D - c_p) B_p), D = sum_p D_p.
      if (!mbar_wait(&bar[kQbAB], tc & 1, ctx, 22)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      constexpr int kHalf = D / 2;
      // workspace slot: A [128][D], B [128][D], D_p [128], c_p [128] (fp32)
      constexpr size_t kSlot = static_cast<size_t>(2) * kTile * D + 2 * kTile;
      float Dfull = 0.f;
      if constexpr (!kGivenD) {
        float Dother = 0.f;
        if (!swap(Dacc, Dother)) { ok = false; break; }
        Dfull = Dacc + Dother;
      }
      if (part < 0) {
        // this row's kHalf outputs, packed to 16-bit as 16-byte chunks, then
        // stored warp-coalesced
        uint4 ch[kHalf / 8];
        const float sD = kGivenD ? 0.f : Dfull - shift;
#pragma unroll
        for (int x = 0; x < kHalf / 32; ++x) {
          uint32_t a[32], bb[32];
          __syncwarp();  // .sync.aligned TMEM access
          tmem_load_32(lane_base + Cfg::kColA + c * kHalf + 32 * x, a);
          if constexpr (!kGivenD) tmem_load_32(lane_base + Cfg::kColB + c * kHalf + 32 * x, bb);
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            float v[8];
#pragma unroll
            for (int z = 0; z < 8; ++z)
              v[z] = kGivenD ? __uint_as_float(a[8 * y + z])
                             : fmaf(-sD, __uint_as_float(bb[8 * y + z]), __uint_as_float(a[8 * y + z]));
            ch[4 * x + y] = make_uint4(Elem<T>::pack(v[0], v[1]), Elem<T>::pack(v[2], v[3]),
                                       Elem<T>::pack(v[4], v[5]), Elem<T>::pack(v[6], v[7]));
          }
        }
        {
          const int row0 = m - lane;  // this warp's first row (query index)
          store_rows_coalesced<kHalf / 8>(
              ch, reinterpret_cast<uint8_t*>(dQ + (static_cast<int64_t>(h) * M + row0) * D + c * kHalf),
              static_cast<size_t>(D) * sizeof(T), lane, M - row0);
        }
        if (!kGivenD && c == 0 && m < M) Dsum[static_cast<int64_t>(h) * M + m] = Dfull;
      } else {
        float* mine = part_ws + static_cast<size_t>(u - um.full) * kSlot;
#pragma unroll
        for (int which = 0; which < (kGivenD ? 1 : 2); ++which) {
#pragma unroll
          for (int x = 0; x < kHalf / 32; ++x) {
            uint32_t a[32];
            __syncwarp();
            tmem_load_32(lane_base + (which == 0 ? Cfg::kColA : Cfg::kColB) + c * kHalf + 32 * x, a);
            float4* dst = reinterpret_cast<float4*>(mine + (static_cast<size_t>(which) * kTile + r) * D +
                                                    c * kHalf + 32 * x);
#pragma unroll
            for (int y = 0; y < 8; ++y)
              dst[y] = make_float4(__uint_as_float(a[4 * y]), __uint_as_float(a[4 * y + 1]),
                                   __uint_as_float(a[4 * y + 2]), __uint_as_float(a[4 * y + 3]));
          }
        }
        if (c == 0) {
          mine[2 * kTile * D + r] = Dfull;
          mine[2 * kTile * D + kTile + r] = shift;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kQbAccEmpty]);
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
// One CTA per (128-row key tile j, head), walking the query tiles i. Items
// take the heads from the last to the first (item t: head H - 1 - t / tiles):
// dq_kernel, which runs just before on the same stream, takes them from the
// first to the last, so the first waves here read the P and dO rows that it
// read last, while they are still in L2. The transposed products keep the
// key index on the TMEM lanes:
//   dP_ij^T = V_j dO_i^T             (A = V_j, B = dO_i, both K-major over d)
//   dS_ij^T = P_ij^T (dP_ij^T - D_i) (dS warps; written back into TMEM, 16-bit)
//   dV_j  += P_ij^T dO_i             (A = P^T, B = dO_i, both MN-major)
//   dK_j  += dS_ij^T Q_i             (A = dS^T from TMEM, B = Q_i MN-major)
// so dS never touches shared memory. The dS warps read P^T as 8x8 transposed
// blocks (ldmatrix.trans) that line up element for element with the
// .16x256b TMEM fragments of dP^T, and store the packed dS^T pairs with
// .16x128b, which is the TS operand layout (lane = key, two queries per
// 32-bit column).
//
// Shared memory (D = 128): V_j 32 KB, P_ij x2 64 KB, dO_i x2 64 KB, Q_i x2
// 64 KB = 224 KB. TMEM: two dP^T/dS^T buffers [0,256) (lane = key, column =
// query), dV [256,256+D), dK [256+D,256+2D) (lane = key, column = d).
//
// Warp roles: 0 TMA for V_j and the P stream; 1 MMA issuer for dP^T (and
// TMEM owner); 2 TMA for dO_i and Q_i; 3 MMA issuer for dV; 4-11 dS warps
// (TMEM lane quarter = warp % 4, query half = (warp - 4) / 4), which also
// write dK_j, dV_j; 12 MMA issuer for dK. A thread between two of its MMA
// groups spends a few hundred cycles on barrier waits and commits even when
// nothing is outstanding, so three issuing threads keep the pipe fed better
// (at D = 128 too: 4.9 % fewer SM cycles at FLUX than dV issued right behind
// dP^T on one thread).
template <int D>
struct DkvCfg {
  static constexpr int kMD = (D / kBoxCols) * kBoxBytes;
  static constexpr int kPT = 2 * kBoxBytes;
  // ring depths: D = 128 fills shared memory with two slots each; D = 64
  // has the room for deeper rings (P 3, dO 4, Q 3)
  static constexpr int kSP = D == 128 ? 2 : 3;  // P_ij slots
  static constexpr int kSD = D == 128 ? 2 : 4;  // dO_i slots
  static constexpr int kSQ = D == 128 ? 2 : 3;  // Q_i slots
  static constexpr int kOffV = 0;
  static constexpr int kOffP = kOffV + kMD;
  static constexpr int kOffdO = kOffP + kSP * kPT;
  static constexpr int kOffQ = kOffdO + kSD * kMD;
  static constexpr int kTileBytes = kOffQ + kSQ * kMD;
  static constexpr int kBarBytes = 512;
  static constexpr int kSmemBytes = kTileBytes + kBarBytes + 1024;
  static constexpr int kDSWarps = 8;
  static constexpr int kFirstDSWarp = 4;
  // warps 1, 3 and kDKWarp issue dP^T, dV and dK, one thread each
  static constexpr int kDKWarp = kFirstDSWarp + kDSWarps;  // dK issuer
  static constexpr int kThreads = 32 * (kDKWarp + 1);
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kNX = D == 128 ? 2 : 3;  // dP^T/dS^T buffers
  static constexpr uint32_t kColX = 0;          // + 128 * buffer
  static constexpr uint32_t kColdV = 128 * kNX;
  static constexpr uint32_t kColdK = kColdV + D;
  static_assert(kColdK + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum DkvBar : int {
  kKbV = 0,
  kKbPFull0 = 1,    // + slot (up to 3)
  kKbPEmpty0 = 4,   // + slot: dV commit + 8 dS warps
  kKbDOFull0 = 7,   // + slot (up to 4)
  kKbDOEmpty0 = 11, // + slot: dP^T and dV commits (one commit after both at D = 128)
  kKbQFull0 = 15,   // + slot (up to 3)
  kKbQEmpty0 = 18,  // + slot
  kKbXFull0 = 21,   // + TMEM buffer (up to 3): dP^T_i computed
  kKbEFull0 = 24,   // + TMEM buffer: dS^T_i written (8 dS warps)
  kKbXFree0 = 27,   // + TMEM buffer: dK_i has read dS^T_i
  kKbAcc = 30,       // dV and dK of an item complete (a commit from each issuer)
  kKbDrain = 31,
  kKbDrain2 = 32,
  kKbVEmpty = 33,    // the dP^T MMAs of an item are done with V_j
  kKbAccEmpty = 34,  // the dS warps have read an item's dV and dK (8 warps)
  kKbDrain3 = 35,    // drain of the dK issuer
  kNumDkvBars = 36,
};
static_assert(kNumDkvBars * 8 + 8 <= 512, "dkv barrier area");

template <typename T, int D>
__global__ void __launch_bounds__(DkvCfg<D>::kThreads, 1)
    dkv_kernel(const __grid_constant__ CUtensorMap tm_Q, const __grid_constant__ CUtensorMap tm_V,
               const __grid_constant__ CUtensorMap tm_dO, const __grid_constant__ CUtensorMap tm_P,
               const float* __restrict__ Dsum, T* __restrict__ dK, T* __restrict__ dV, int M, int N,
               int H, UnitMap um, float* __restrict__ part_ws,
               KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = DkvCfg<D>;
  constexpr int kEpi = Cfg::kDSWarps;
  constexpr int NX = Cfg::kNX;
  constexpr int SP = Cfg::kSP, SD = Cfg::kSD, SQ = Cfg::kSQ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumDkvBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt = (M + kTile - 1) / kTile;
  const int ntk = (N + kTile - 1) / kTile;
  // work items (key tile, head), head-major, walked as work units (um): a
  // unit is an item's query tiles [lo, hi)

  if (threadIdx.x == 0) {
    mbar_init(&bar[kKbV], 1);
    mbar_init(&bar[kKbVEmpty], 1);
    mbar_init(&bar[kKbAccEmpty], kEpi);
    for (int s = 0; s < SP; ++s) {
      mbar_init(&bar[kKbPFull0 + s], 1);
      mbar_init(&bar[kKbPEmpty0 + s], 1 + kEpi);
    }
    for (int s = 0; s < SD; ++s) {
      mbar_init(&bar[kKbDOFull0 + s], 1);
      mbar_init(&bar[kKbDOEmpty0 + s], 2);  // dP^T and dV commits
    }
    for (int s = 0; s < SQ; ++s) {
      mbar_init(&bar[kKbQFull0 + s], 1);
      mbar_init(&bar[kKbQEmpty0 + s], 1);
    }
    for (int s = 0; s < Cfg::kNX; ++s) {
      mbar_init(&bar[kKbXFull0 + s], 1);
      mbar_init(&bar[kKbEFull0 + s], kEpi);
      mbar_init(&bar[kKbXFree0 + s], 1);
    }
    mbar_init(&bar[kKbAcc], 2);
    mbar_init(&bar[kKbDrain], 1);
    mbar_init(&bar[kKbDrain2], 1);
    mbar_init(&bar[kKbDrain3], 1);
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

  // Every role walks the same work units: u = blockIdx.x, + gridDim.x, ...
  // Shared-memory rings, TMEM buffers and their barrier phases continue
  // across units (global step counter g over (unit, query tile)).
  if (warp == 0) {
    // ---- TMA producer: per item V_j (once the previous item's dP^T MMAs are
    // done), then the P stream (2 slots).
    if (lane == 0) {
      tma_prefetch_desc(&tm_V);
      tma_prefetch_desc(&tm_P);
      const uint64_t pol_p = l2_policy_evict_first();
      const uint64_t pol_v = l2_policy_evict_normal();
      int g = 0, issued = 0, nv = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x) {
        int t, lo, hi, part;
        um.get(u, mt, t, lo, hi, part);
        const int hl = t / ntk;
        const int n0 = (t - hl * ntk) * kTile;
        const int h = H - 1 - hl;
        if (nv > 0 && !mbar_wait(&bar[kKbVEmpty], (nv - 1) & 1, ctx, 32)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar[kKbV], Cfg::kMD);
#pragma unroll
        for (int b = 0; b < D / kBoxCols; ++b)
          tma_load_3d(smem + Cfg::kOffV + b * kBoxBytes, &tm_V, &bar[kKbV], b * kBoxCols, n0, h, pol_v);
        ++nv;
        for (int i = lo; i < hi; ++i, ++g) {
          const int s = g % SP;
          const int r = g / SP;
          if (r > 0 && !mbar_wait(&bar[kKbPEmpty0 + s], (r - 1) & 1, ctx, 30)) { ok = false; break; }
          uint8_t* dst = smem + Cfg::kOffP + s * Cfg::kPT;
          mbar_arrive_expect_tx(&bar[kKbPFull0 + s], Cfg::kPT);
          tma_load_3d(dst, &tm_P, &bar[kKbPFull0 + s], n0, i * kTile, h, pol_p);
          tma_load_3d(dst + kBoxBytes, &tm_P, &bar[kKbPFull0 + s], n0 + kBoxCols, i * kTile, h, pol_p);
          ++issued;
        }
      }
      if (*abort_flag) {
        if (nv > 0) mbar_wait_drain(&bar[kKbV], (nv - 1) & 1, timeout_ns);
        for (int i = (issued > SP ? issued - SP : 0); i < issued; ++i)
          mbar_wait_drain(&bar[kKbPFull0 + i % SP], (i / SP) & 1, timeout_ns);
      }
    }
  } else if (warp == 2) {
    // ---- TMA producer for the L2-resident operands dO_i and Q_i (two slots
    // each; every key-tile CTA of the head reads them). Polls both "empty"
    // barriers without blocking and issues whichever load can go (no L2
    // prefetch ahead, as in the other producers).
    if (lane == 0) {
      tma_prefetch_desc(&tm_dO);
      tma_prefetch_desc(&tm_Q);
      const uint64_t pol = l2_policy_evict_last();
      // cursors over this CTA's sequence of (unit, query tile): the next dO
      // load and the next Q load
      struct Cursor {
        int u, i, hi, h;
      };
      auto start = [&](Cursor& c, int u) {
        c.u = u;
        if (u < um.units) {
          int t, lo, hi, part;
          um.get(u, mt, t, lo, hi, part);
          c.i = lo;
          c.hi = hi;
          c.h = H - 1 - t / ntk;
        }
      };
      auto advance = [&](Cursor& c) {
        if (++c.i >= c.hi) start(c, c.u + static_cast<int>(gridDim.x));
      };
      Cursor cd, cq;
      start(cd, blockIdx.x);
      start(cq, blockIdx.x);
      int next_do = 0, next_q = 0;  // loads issued (ring phases)
      uint64_t t_last = global_timer_ns();
      bool failed = false;
      while ((cd.u < um.units || cq.u < um.units) && !failed) {
        bool progressed = false;
        if (cd.u < um.units && (next_do < SD || mbar_poll(&bar[kKbDOEmpty0 + next_do % SD], ((next_do / SD) - 1) & 1))) {
          const int s = next_do % SD;
          mbar_arrive_expect_tx(&bar[kKbDOFull0 + s], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffdO + s * Cfg::kMD + b * kBoxBytes, &tm_dO, &bar[kKbDOFull0 + s],
                        b * kBoxCols, cd.i * kTile, cd.h, pol);
          advance(cd);
          ++next_do;
          progressed = true;
        }
        if (cq.u < um.units && (next_q < SQ || mbar_poll(&bar[kKbQEmpty0 + next_q % SQ], ((next_q / SQ) - 1) & 1))) {
          const int s = next_q % SQ;
          mbar_arrive_expect_tx(&bar[kKbQFull0 + s], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffQ + s * Cfg::kMD + b * kBoxBytes, &tm_Q, &bar[kKbQFull0 + s],
                        b * kBoxCols, cq.i * kTile, cq.h, pol);
          advance(cq);
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
        for (int i = (next_do > SD ? next_do - SD : 0); i < next_do; ++i)
          mbar_wait_drain(&bar[kKbDOFull0 + i % SD], (i / SD) & 1, timeout_ns);
        for (int i = (next_q > SQ ? next_q - SQ : 0); i < next_q; ++i)
          mbar_wait_drain(&bar[kKbQFull0 + i % SQ], (i / SQ) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == 3 || warp == Cfg::kDKWarp) {
    // ---- MMA issuers, one thread per product (the others keep the tensor
    // pipe fed while one waits). Warp 1: dP^T_i into TMEM buffer i % NX;
    // warp 3: dV_j += P_ij^T dO_i; kDKWarp: dK_j += dS_ij^T Q_i. dO_i's
    // ring slot is released by the dP^T and dV commits.
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      constexpr uint32_t id_dP = make_idesc_f16<kB>(kTile, kTile, false, false);
      constexpr uint32_t id_dV = make_idesc_f16<kB>(kTile, D, true, true);
      constexpr uint32_t id_dK = make_idesc_f16<kB>(kTile, D, false, true);
      const uint64_t dVt = make_sw128_desc(smem_u32(smem + Cfg::kOffV), 16, 1024);
      bool ok = true;
      if (warp == 1) {
        int g = 0, tc = 0;
        for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
        int t, lo, hi, part;
        um.get(u, mt, t, lo, hi, part);
        if (!mbar_wait(&bar[kKbV], tc & 1, ctx, 45)) { ok = false; break; }
        for (int i = lo; i < hi; ++i, ++g) {
          const int s = g % SD;
          const uint64_t ddO = make_sw128_desc(smem_u32(smem + Cfg::kOffdO + s * Cfg::kMD), 16, 1024);
          if (!mbar_wait(&bar[kKbDOFull0 + s], (g / SD) & 1, ctx, 40)) { ok = false; break; }
          // buffer g % 2 is free once dK has read dS^T of step g - 2 from it
          const int x = g % NX;
          if (g >= NX && !mbar_wait(&bar[kKbXFree0 + x], ((g / NX) - 1) & 1, ctx, 41)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
            umma_f16_ss(tmem + Cfg::kColX + 128 * x, desc_advance(dVt, off), desc_advance(ddO, off), id_dP,
                        k > 0 ? 1u : 0u);
          }
          umma_commit(&bar[kKbXFull0 + x]);
          umma_commit(&bar[kKbDOEmpty0 + s]);
        }
        if (ok) umma_commit(&bar[kKbVEmpty]);  // V_j consumed
        }
        if (!ok) {
          umma_commit(&bar[kKbDrain]);
          mbar_wait_drain(&bar[kKbDrain], 0, timeout_ns);
        }
      } else if (warp == 3) {
        int g = 0, tc = 0;
        for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
          int t, lo, hi, part;
          um.get(u, mt, t, lo, hi, part);
          // dV of the previous unit must have been read out first
          if (tc > 0 && !mbar_wait(&bar[kKbAccEmpty], (tc - 1) & 1, ctx, 47)) { ok = false; break; }
          for (int i = lo; i < hi; ++i, ++g) {
            const int sp = g % SP, sd = g % SD;
            // dV += P_ij^T dO_i : A = P^T (MN-major, M = key), B = dO_i (MN-major, N = d).
            if (!mbar_wait(&bar[kKbPFull0 + sp], (g / SP) & 1, ctx, 42)) { ok = false; break; }
            if (!mbar_wait(&bar[kKbDOFull0 + sd], (g / SD) & 1, ctx, 46)) { ok = false; break; }
            tc_fence_after();
            const uint64_t ddO = make_sw128_desc(smem_u32(smem + Cfg::kOffdO + sd * Cfg::kMD), kBoxBytes, 1024);
            const uint64_t dP = make_sw128_desc(smem_u32(smem + Cfg::kOffP + sp * Cfg::kPT), kBoxBytes, 1024);
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              umma_f16_ss(tmem + Cfg::kColdV, desc_advance(dP, k * 2048), desc_advance(ddO, k * 2048), id_dV,
                          (i > lo || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[kKbDOEmpty0 + sd]);
            umma_commit(&bar[kKbPEmpty0 + sp]);
          }
          if (ok) umma_commit(&bar[kKbAcc]);
        }
        if (!ok) {
          umma_commit(&bar[kKbDrain2]);
          mbar_wait_drain(&bar[kKbDrain2], 0, timeout_ns);
        }
      } else {
        int g = 0, tc = 0;
        for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
          int t, lo, hi, part;
          um.get(u, mt, t, lo, hi, part);
          // dK of the previous unit must have been read out first
          if (tc > 0 && !mbar_wait(&bar[kKbAccEmpty], (tc - 1) & 1, ctx, 55)) { ok = false; break; }
          for (int i = lo; i < hi; ++i, ++g) {
            const int s = g % SQ;
            // dK += dS^T Q_i : A = dS^T from TMEM buffer g % NX (16 queries =
            // 8 packed columns per step), B = Q_i (MN-major, N = d).
            if (!mbar_wait(&bar[kKbQFull0 + s], (g / SQ) & 1, ctx, 43)) { ok = false; break; }
            if (!mbar_wait(&bar[kKbEFull0 + g % NX], (g / NX) & 1, ctx, 44)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dQd = make_sw128_desc(smem_u32(smem + Cfg::kOffQ + s * Cfg::kMD), kBoxBytes, 1024);
            const uint32_t tS = tmem + Cfg::kColX + 128 * (g % NX);
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              umma_f16_ts(tmem + Cfg::kColdK, tS + (k >> 2) * 64 + (k & 3) * 8,
                          desc_advance(dQd, k * 2048), id_dK, (i > lo || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[kKbQEmpty0 + s]);
            umma_commit(&bar[kKbXFree0 + g % NX]);
          }
          if (ok) umma_commit(&bar[kKbAcc]);
        }
        if (!ok) {
          umma_commit(&bar[kKbDrain3]);
          mbar_wait_drain(&bar[kKbDrain3], 0, timeout_ns);
        }
      }
    }
  } else if (warp >= Cfg::kFirstDSWarp && warp < Cfg::kFirstDSWarp + Cfg::kDSWarps) {
    // ---- dS warps. Warp w owns TMEM lane quarter qq = w % 4 (keys
    // 32qq..32qq+31 of the tile, as two 16-lane halves) and query half c
    // (queries 64c..64c+63 of each query tile). In the .16x256b fragment,
    // thread t holds keys t/4 and 8 + t/4 of a half and queries
    // 8 blk + 2 (t%4) + {0,1} of each 8-query block blk.
    const int qq = warp & 3;
    const int c = (warp - Cfg::kFirstDSWarp) >> 2;
    const uint32_t lq = static_cast<uint32_t>(lane & 3);
    bool ok = true;
    int g = 0, tc = 0;
    for (int u = blockIdx.x; u < um.units && ok; u += gridDim.x, ++tc) {
    int t, lo, hi, part;
    um.get(u, mt, t, lo, hi, part);
    const int hl = t / ntk;
    const int n0 = (t - hl * ntk) * kTile;
    const int h = H - 1 - hl;
    for (int i = lo; i < hi; ++i, ++g) {
      const int s = g % SP;  // P slot of this step
      // D for this thread's 16 queries (rows of the query tile past M read 0)
      float Dv[16];
      {
        const int64_t drow = static_cast<int64_t>(h) * M;
        const int q0 = i * kTile + 64 * c + 2 * static_cast<int>(lq);
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) {
          const int q = q0 + 8 * blk;
          Dv[2 * blk] = q < M ? __ldg(Dsum + drow + q) : 0.f;
          Dv[2 * blk + 1] = q + 1 < M ? __ldg(Dsum + drow + q + 1) : 0.f;
        }
      }
      const int x = g % NX;  // TMEM buffer of this step
      if (!mbar_wait(&bar[kKbXFull0 + x], (g / NX) & 1, ctx, 50)) { ok = false; break; }
      if (!mbar_wait(&bar[kKbPFull0 + s], (g / SP) & 1, ctx, 51)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      const uint32_t sP = smem_u32(smem + Cfg::kOffP + s * Cfg::kPT);
      const uint32_t tX = tmem + Cfg::kColX + 128 * x + 64 * c;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t lane_addr = static_cast<uint32_t>(32 * qq + 16 * hh) << 16;
        uint32_t dp[32];
        tmem_load_16x256b_x8(tX + lane_addr, dp);
        // P^T fragments: for query pair p (queries 16p..16p+15 of the half),
        // matrices (queries +0..7 | +8..15) x (keys +0..7 | +8..15).
        uint32_t pf[4][4];
        {
          const int m = lane >> 3, rr = lane & 7;
          const int key = 32 * qq + 16 * hh + 8 * (m >> 1);  // key within the tile
          const uint32_t box = sP + static_cast<uint32_t>(key >> 6) * kBoxBytes;
          const uint32_t chunk = static_cast<uint32_t>((key & 63) >> 3);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint32_t row = static_cast<uint32_t>(64 * c + 16 * p + rr + 8 * (m & 1));
            ldmatrix_x4_trans(box + row * 128u + ((chunk ^ (row & 7u)) << 4), pf[p]);
          }
        }
        uint32_t ds[16];
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) {
          const int p = blk >> 1, odd = blk & 1;
          const float2 dv = make_float2(-Dv[2 * blk], -Dv[2 * blk + 1]);
          const float2 ptop = Elem<T>::unpack(pf[p][odd]);
          const float2 pbot = Elem<T>::unpack(pf[p][2 + odd]);
          const float2 gtop = make_float2(__uint_as_float(dp[4 * blk]), __uint_as_float(dp[4 * blk + 1]));
          const float2 gbot = make_float2(__uint_as_float(dp[4 * blk + 2]), __uint_as_float(dp[4 * blk + 3]));
          const float2 stop = mul_f32x2(ptop, add_f32x2(gtop, dv));
          const float2 sbot = mul_f32x2(pbot, add_f32x2(gbot, dv));
          ds[2 * blk] = Elem<T>::pack(stop.x, stop.y);
          ds[2 * blk + 1] = Elem<T>::pack(sbot.x, sbot.y);
        }
        // packed dS^T of the half's 64 queries -> first 32 columns of its region
        tmem_store_16x128b_x8(tX + lane_addr, ds);
      }
      tmem_store_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[kKbEFull0 + x]);
        mbar_arrive(&bar[kKbPEmpty0 + s]);
      }
    }
    if (!ok) break;
    // final dV_j and dK_j rows (lane = key row) -> 16-bit outputs (a whole
    // item) or fp32 partials in the workspace (a part of a tail item), then
    // hand the accumulators back to the issuers
    if (!mbar_wait(&bar[kKbAcc], tc & 1, ctx, 53)) { ok = false; break; }
    const int r = qq * 32 + lane;
    constexpr int kHalf = D / 2;
    constexpr size_t kSlot = static_cast<size_t>(2) * kTile * D;  // floats per workspace slot
    {
      __syncwarp();
      tc_fence_after();
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(qq * 32) << 16);
      float* mine = part >= 0 ? part_ws + static_cast<size_t>(u - um.full) * kSlot : nullptr;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = (which == 0 ? Cfg::kColdV : Cfg::kColdK) + c * kHalf;
        uint4 ch[kHalf / 8];  // a whole item's row, packed to 16-bit
#pragma unroll
        for (int x = 0; x < kHalf / 32; ++x) {
          uint32_t v[32];
          __syncwarp();  // .sync.aligned TMEM access: the warp reconverges after the
                         // row-guarded stores of the previous iteration
          tmem_load_32(lane_base + col + x * 32, v);
          if (part < 0) {
#pragma unroll
            for (int y = 0; y < 4; ++y)
              ch[4 * x + y] = make_uint4(
                  Elem<T>::pack(__uint_as_float(v[8 * y]), __uint_as_float(v[8 * y + 1])),
                  Elem<T>::pack(__uint_as_float(v[8 * y + 2]), __uint_as_float(v[8 * y + 3])),
                  Elem<T>::pack(__uint_as_float(v[8 * y + 4]), __uint_as_float(v[8 * y + 5])),
                  Elem<T>::pack(__uint_as_float(v[8 * y + 6]), __uint_as_float(v[8 * y + 7])));
          } else {
            float4* dst = reinterpret_cast<float4*>(mine + (static_cast<size_t>(which) * kTile + r) * D +
                                                    c * kHalf + 32 * x);
#pragma unroll
            for (int y = 0; y < 8; ++y)
              dst[y] = make_float4(__uint_as_float(v[4 * y]), __uint_as_float(v[4 * y + 1]),
                                   __uint_as_float(v[4 * y + 2]), __uint_as_float(v[4 * y + 3]));
          }
        }
        if (part < 0) {
          __syncwarp();
          const int row0 = n0 + qq * 32;  // this warp's first row (key index)
          store_rows_coalesced<kHalf / 8>(
              ch,
              reinterpret_cast<uint8_t*>((which == 0 ? dV : dK) + (static_cast<int64_t>(h) * N + row0) * D +
                                         c * kHalf),
              static_cast<size_t>(D) * sizeof(T), lane, N - row0);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kKbAccEmpty]);
    }
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

// ========================================================== combine kernels
// The parts of split tail items leave fp32 partials in workspace slots
// (slot = unit - um.full; the parts of tail item k are slots
// k * parts .. k * parts + parts - 1). These kernels, stream-ordered after the
// main kernel, add them up in part order and write the 16-bit outputs: one
// thread per (tail item, row, 8 columns), reading every part's values before
// adding any (independent, coalesced L2 reads).
constexpr int kCombineThreads = 256;

// dq slot: A [128][D], B [128][D], D_p [128], c_p [128].
// dQ = sum_p A_p - (D - c_p) B_p with D = sum_p D_p, also written to Dsum
// (D given: dQ = sum_p A_p).
template <typename T, int D, bool kGivenD>
__global__ void __launch_bounds__(kCombineThreads)
    dq_combine_kernel(const float* __restrict__ part_ws, UnitMap um, int M, T* __restrict__ dQ,
                      float* __restrict__ Dsum) {
  constexpr int kChunks = D / 8;
  constexpr size_t kSlot = static_cast<size_t>(2) * kTile * D + 2 * kTile;
  const int mt = (M + kTile - 1) / kTile;
  const int tail = (um.units - um.full) / um.parts;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * kCombineThreads + threadIdx.x;
  const int x = static_cast<int>(idx % kChunks);
  const int r = static_cast<int>((idx / kChunks) % kTile);
  const int64_t k = idx / (kChunks * kTile);
  if (k >= tail) return;
  const int item = um.full + static_cast<int>(k);
  const int h = item / mt;
  const int m = (item - h * mt) * kTile + r;
  if (m >= M) return;
  const float* first = part_ws + static_cast<size_t>(k) * um.parts * kSlot;
  float Dp[kMaxParts], cp[kMaxParts];
  float4 a[kMaxParts][2], b[kMaxParts][2];
#pragma unroll
  for (int p = 0; p < kMaxParts; ++p) {
    if (p < um.parts) {
      const float* sp = first + p * kSlot;
      const float4* pa = reinterpret_cast<const float4*>(sp + static_cast<size_t>(r) * D + 8 * x);
      a[p][0] = __ldcg(pa);
      a[p][1] = __ldcg(pa + 1);
      if constexpr (!kGivenD) {
        const float4* pb = reinterpret_cast<const float4*>(sp + static_cast<size_t>(kTile + r) * D + 8 * x);
        b[p][0] = __ldcg(pb);
        b[p][1] = __ldcg(pb + 1);
        Dp[p] = __ldcg(sp + 2 * kTile * D + r);
        cp[p] = __ldcg(sp + 2 * kTile * D + kTile + r);
      }
    }
  }
  float Dtot = 0.f;
  if constexpr (!kGivenD) {
#pragma unroll
    for (int p = 0; p < kMaxParts; ++p)
      if (p < um.parts) Dtot += Dp[p];
  }
  float v[8];
#pragma unroll
  for (int y = 0; y < 8; ++y) v[y] = 0.f;
#pragma unroll
  for (int p = 0; p < kMaxParts; ++p) {
    if (p < um.parts) {
      v[0] += a[p][0].x; v[1] += a[p][0].y; v[2] += a[p][0].z; v[3] += a[p][0].w;
      v[4] += a[p][1].x; v[5] += a[p][1].y; v[6] += a[p][1].z; v[7] += a[p][1].w;
      if constexpr (!kGivenD) {
        const float sD = Dtot - cp[p];
        v[0] = fmaf(-sD, b[p][0].x, v[0]); v[1] = fmaf(-sD, b[p][0].y, v[1]);
        v[2] = fmaf(-sD, b[p][0].z, v[2]); v[3] = fmaf(-sD, b[p][0].w, v[3]);
        v[4] = fmaf(-sD, b[p][1].x, v[4]); v[5] = fmaf(-sD, b[p][1].y, v[5]);
        v[6] = fmaf(-sD, b[p][1].z, v[6]); v[7] = fmaf(-sD, b[p][1].w, v[7]);
      }
    }
  }
  *reinterpret_cast<uint4*>(dQ + (static_cast<int64_t>(h) * M + m) * D + 8 * x) =
      make_uint4(Elem<T>::pack(v[0], v[1]), Elem<T>::pack(v[2], v[3]), Elem<T>::pack(v[4], v[5]),
                 Elem<T>::pack(v[6], v[7]));
  if (!kGivenD && x == 0) Dsum[static_cast<int64_t>(h) * M + m] = Dtot;
}

// dkv slot: dV [128][D], dK [128][D]; each is the sum of its parts.
template <typename T, int D>
__global__ void __launch_bounds__(kCombineThreads)
    dkv_combine_kernel(const float* __restrict__ part_ws, UnitMap um, int N, T* __restrict__ dK,
                       T* __restrict__ dV) {
  constexpr int kChunks = D / 8;
  constexpr size_t kSlot = static_cast<size_t>(2) * kTile * D;
  const int ntk = (N + kTile - 1) / kTile;
  const int tail = (um.units - um.full) / um.parts;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * kCombineThreads + threadIdx.x;
  const int x = static_cast<int>(idx % kChunks);
  const int64_t row = idx / kChunks;           // (tail item, which, key row)
  const int r = static_cast<int>(row % kTile);
  const int which = static_cast<int>((row / kTile) % 2);
  const int64_t k = row / (2 * kTile);
  if (k >= tail) return;
  const int item = um.full + static_cast<int>(k);
  const int hl = item / ntk;
  const int n = (item - hl * ntk) * kTile + r;
  const int h = (um.full + tail) / ntk - 1 - hl;  // heads last to first, as in dkv_kernel
  if (n >= N) return;
  const float* src = part_ws + static_cast<size_t>(k) * um.parts * kSlot +
                     (static_cast<size_t>(which) * kTile + r) * D + 8 * x;
  float4 f[kMaxParts][2];
#pragma unroll
  for (int p = 0; p < kMaxParts; ++p) {
    if (p < um.parts) {
      const float4* sp = reinterpret_cast<const float4*>(src + p * kSlot);
      f[p][0] = __ldcg(sp);
      f[p][1] = __ldcg(sp + 1);
    }
  }
  float4 a0 = f[0][0], a1 = f[0][1];
#pragma unroll
  for (int p = 1; p < kMaxParts; ++p) {
    if (p < um.parts) {
      a0.x += f[p][0].x; a0.y += f[p][0].y; a0.z += f[p][0].z; a0.w += f[p][0].w;
      a1.x += f[p][1].x; a1.y += f[p][1].y; a1.z += f[p][1].z; a1.w += f[p][1].w;
    }
  }
  T* out = (which == 0 ? dV : dK) + (static_cast<int64_t>(h) * N + n) * D + 8 * x;
  *reinterpret_cast<uint4*>(out) = make_uint4(Elem<T>::pack(a0.x, a0.y), Elem<T>::pack(a0.z, a0.w),
                                              Elem<T>::pack(a1.x, a1.y), Elem<T>::pack(a1.z, a1.w));
}

}  // namespace fmha_sm100
