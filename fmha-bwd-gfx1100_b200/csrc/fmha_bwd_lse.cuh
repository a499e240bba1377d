// Attention backward that recomputes P on chip from Q, K and the row
// log-sum-exp instead of reading a materialised P (the FlashAttention form of
// the backward). Inputs per head: Q, dO [M][d]; K, V [N][d]; O [M][d] (the
// forward output); LSE [M] fp32 with
//     LSE_m = log sum_n exp(scale * Q_m . K_n),   P = exp(scale * Q K^T - LSE).
// Outputs (the gradients of the scaled-score attention):
//     D = rowsum(dO * O),  dS = P * (dP - D),  dP = dO V^T,
//     dQ = scale * dS K,   dK = scale * dS^T Q,  dV = P^T dO.
// With scale = 1 and O = P V this is fmha_bwd_full_py applied to
// P = exp(Q K^T - LSE), without the M x N x 2-byte P in memory.
//
// Three launches on one stream: rowsum_do_o_kernel (D, fp32), then
// dq_lse_kernel and dkv_lse_kernel, each a persistent variant of the
// corresponding P-reading kernel in which the P stream is replaced by an
// extra MMA (S = Q K^T, or S^T = K Q^T) and an exp2 in the epilogue.
#pragma once

#include "fmha_bwd_launch.cuh"

namespace fmha_sm100 {

constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the SFU (PTX ex2.approx.ftz.f32: relative error about 2^-22,
// flushes subnormals; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ======================================================== rowsum_do_o_kernel
// Dsum[row] = sum_k dO[row][k] O[row][k] in fp32, one row per D / 8 threads
// (16-byte chunks), rows = H * M.
template <typename T, int D>
__global__ void __launch_bounds__(256)
    rowsum_do_o_kernel(const T* __restrict__ dO, const T* __restrict__ O, float* __restrict__ Dsum,
                       int64_t rows) {
  constexpr int kPerRow = D / 8;  // threads per row
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (256 / kPerRow) + threadIdx.x / kPerRow;
  const int chunk = threadIdx.x % kPerRow;
  float acc = 0.f;
  if (row < rows) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(dO + row * D) + chunk);
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(O + row * D) + chunk);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 x = Elem<T>::unpack(aw[t]), y = Elem<T>::unpack(bw[t]);
      acc = fmaf(x.x, y.x, acc);
      acc = fmaf(x.y, y.y, acc);
    }
  }
#pragma unroll
  for (int o = kPerRow / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o, kPerRow);
  if (row < rows && chunk == 0) Dsum[row] = acc;
}

// ============================================================= dq_lse_kernel
// Persistent, one CTA per SM walking (128-row query tile i, head) items,
// head-major. Q_i and dO_i stay in shared memory for the item; K_j and V_j
// stream through rings. Per key tile j:
//   S_ij  = Q_i K_j^T        (SS MMA into TMEM buffer S_(g%2))
//   dP_ij = dO_i V_j^T       (SS MMA into the dP buffer)
//   dS    = P (dP - D),  P = 2^(S scale log2e - LSE log2e)   (epilogue;
//           16-bit dS written over the first 32 columns of each 64-column
//           half of S_(g%2))
//   A_i  += dS K_j           (TS MMA, A operand from TMEM)
// and finally dQ_i = scale A_i. D is an input (rowsum_do_o_kernel), so no
// second accumulator is needed. Rows of K_j past N are zero-filled by TMA,
// so the P values of those keys (finite) contribute nothing.
//
// Shared memory (D = 128): Q_i 32 KB, dO_i 32 KB, K_j x2, V_j x2 = 192 KB.
// TMEM: S0 [0,128), S1 [128,256), dP [256,384), A [384,384+D).
// Warps: 0 TMA producer; 1 MMA issuer for S and dP (TMEM owner); 2-9
// epilogue (lane quarter = warp % 4, key half = (warp - 2) / 4); 10 MMA
// issuer for A.
template <int D>
struct DqLseCfg {
  static constexpr int kMD = (D / kBoxCols) * kBoxBytes;
  static constexpr int kSK = D == 128 ? 2 : 4;
  static constexpr int kSV = D == 128 ? 2 : 4;
  static constexpr int kOffQ = 0;
  static constexpr int kOffdO = kMD;
  static constexpr int kOffK = 2 * kMD;
  static constexpr int kOffV = kOffK + kSK * kMD;
  static constexpr int kOffBar = kOffV + kSV * kMD;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kOffBar + kBarBytes + 1024;
  static constexpr int kEpiWarps = 8;
  static constexpr int kFirstEpiWarp = 2;
  static constexpr int kAWarp = kFirstEpiWarp + kEpiWarps;
  static constexpr int kThreads = 32 * (kAWarp + 1);
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColS = 0;  // + 128 * buffer
  static constexpr uint32_t kColdP = 256;
  static constexpr uint32_t kColA = 384;
  static_assert(kColA + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum DqLseBar : int {
  kLqQFull = 0,    // Q_i and dO_i landed
  kLqQEmpty = 1,   // the S and dP MMAs of the item are done with Q_i, dO_i
  kLqKFull0 = 2,   // + slot (up to 4)
  kLqKEmpty0 = 6,  // + slot
  kLqVFull0 = 10,  // + slot
  kLqVEmpty0 = 14, // + slot
  kLqSFull0 = 18,  // + S buffer (2)
  kLqEFull0 = 20,  // + S buffer: dS written (8 epilogue warps)
  kLqSFree0 = 22,  // + S buffer: A has read dS
  kLqdPFull = 24,
  kLqdPRead = 25,  // the epilogue has read dP (8 warps)
  kLqAcc = 26,     // A of an item complete
  kLqAccEmpty = 27,
  kLqDrain = 28,
  kLqDrain2 = 29,
  kNumDqLseBars = 30,
};
static_assert(kNumDqLseBars * 8 + 8 <= 256, "dq_lse barrier area");

template <typename T, int D>
__global__ void __launch_bounds__(DqLseCfg<D>::kThreads, 1)
    dq_lse_kernel(const __grid_constant__ CUtensorMap tm_Q, const __grid_constant__ CUtensorMap tm_K,
                  const __grid_constant__ CUtensorMap tm_V, const __grid_constant__ CUtensorMap tm_dO,
                  const float* __restrict__ LSE, const float* __restrict__ Dsum, T* __restrict__ dQ,
                  int M, int N, int H, float scale, KernelStatus* status, uint64_t timeout_ns) {
  using Cfg = DqLseCfg<D>;
  constexpr int SK = Cfg::kSK, SV = Cfg::kSV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumDqLseBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt = (M + kTile - 1) / kTile;
  const int nt = (N + kTile - 1) / kTile;
  const int tiles = mt * H;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kLqQFull], 1);
    mbar_init(&bar[kLqQEmpty], 1);
    for (int s = 0; s < SK; ++s) {
      mbar_init(&bar[kLqKFull0 + s], 1);
      mbar_init(&bar[kLqKEmpty0 + s], 1);
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(&bar[kLqVFull0 + s], 1);
      mbar_init(&bar[kLqVEmpty0 + s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar[kLqSFull0 + b], 1);
      mbar_init(&bar[kLqEFull0 + b], Cfg::kEpiWarps);
      mbar_init(&bar[kLqSFree0 + b], 1);
    }
    mbar_init(&bar[kLqdPFull], 1);
    mbar_init(&bar[kLqdPRead], Cfg::kEpiWarps);
    mbar_init(&bar[kLqAcc], 1);
    mbar_init(&bar[kLqAccEmpty], Cfg::kEpiWarps);
    mbar_init(&bar[kLqDrain], 1);
    mbar_init(&bar[kLqDrain2], 1);
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
    // ---- TMA producer: per item Q_i and dO_i (once the previous item's S
    // and dP MMAs are done), then K_j and V_j for every key tile.
    if (lane == 0) {
      tma_prefetch_desc(&tm_Q);
      tma_prefetch_desc(&tm_K);
      tma_prefetch_desc(&tm_V);
      tma_prefetch_desc(&tm_dO);
      const uint64_t pol_q = l2_policy_evict_normal();
      const uint64_t pol_kv = l2_policy_evict_last();
      int g = 0, nQ = 0, nK = 0, nV = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int h = t / mt;
        const int m0 = (t - h * mt) * kTile;
        if (nQ > 0 && !mbar_wait(&bar[kLqQEmpty], (nQ - 1) & 1, ctx, 101)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar[kLqQFull], 2 * Cfg::kMD);
#pragma unroll
        for (int b = 0; b < D / kBoxCols; ++b) {
          tma_load_3d(smem + Cfg::kOffQ + b * kBoxBytes, &tm_Q, &bar[kLqQFull], b * kBoxCols, m0, h, pol_q);
          tma_load_3d(smem + Cfg::kOffdO + b * kBoxBytes, &tm_dO, &bar[kLqQFull], b * kBoxCols, m0, h, pol_q);
        }
        ++nQ;
        for (int j = 0; j < nt; ++j, ++g) {
          if (g >= SK && !mbar_wait(&bar[kLqKEmpty0 + g % SK], ((g / SK) - 1) & 1, ctx, 102)) { ok = false; break; }
          {
            uint64_t* fb = &bar[kLqKFull0 + g % SK];
            uint8_t* dst = smem + Cfg::kOffK + (g % SK) * Cfg::kMD;
            mbar_arrive_expect_tx(fb, Cfg::kMD);
#pragma unroll
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_load_3d(dst + b * kBoxBytes, &tm_K, fb, b * kBoxCols, j * kTile, h, pol_kv);
            ++nK;
          }
          if (g >= SV && !mbar_wait(&bar[kLqVEmpty0 + g % SV], ((g / SV) - 1) & 1, ctx, 103)) { ok = false; break; }
          {
            uint64_t* fb = &bar[kLqVFull0 + g % SV];
            uint8_t* dst = smem + Cfg::kOffV + (g % SV) * Cfg::kMD;
            mbar_arrive_expect_tx(fb, Cfg::kMD);
#pragma unroll
            for (int b = 0; b < D / kBoxCols; ++b)
              tma_load_3d(dst + b * kBoxBytes, &tm_V, fb, b * kBoxCols, j * kTile, h, pol_kv);
            ++nV;
          }
        }
      }
      if (*abort_flag) {
        if (nQ > 0) mbar_wait_drain(&bar[kLqQFull], (nQ - 1) & 1, timeout_ns);
        for (int j = (nK > SK ? nK - SK : 0); j < nK; ++j)
          mbar_wait_drain(&bar[kLqKFull0 + j % SK], (j / SK) & 1, timeout_ns);
        for (int j = (nV > SV ? nV - SV : 0); j < nV; ++j)
          mbar_wait_drain(&bar[kLqVFull0 + j % SV], (j / SV) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == Cfg::kAWarp) {
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      // S = Q_i K_j^T and dP = dO_i V_j^T: A and B K-major over d
      constexpr uint32_t id_SS = make_idesc_f16<kB>(kTile, kTile, false, false);
      // A += dS K_j: A = dS from TMEM, B = K_j [key][d] MN-major
      constexpr uint32_t id_A = make_idesc_f16<kB>(kTile, D, false, true);
      const uint64_t dQd = make_sw128_desc(smem_u32(smem + Cfg::kOffQ), 16, 1024);
      const uint64_t ddO = make_sw128_desc(smem_u32(smem + Cfg::kOffdO), 16, 1024);
      const uint32_t sK0 = smem_u32(smem + Cfg::kOffK);
      const uint32_t sV0 = smem_u32(smem + Cfg::kOffV);
      bool ok = true;
      int g = 0, tc = 0;
      if (warp == 1) {
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
          if (!mbar_wait(&bar[kLqQFull], tc & 1, ctx, 110)) { ok = false; break; }
          for (int j = 0; j < nt; ++j, ++g) {
            const int b = g & 1;
            if (!mbar_wait(&bar[kLqKFull0 + g % SK], (g / SK) & 1, ctx, 111)) { ok = false; break; }
            // S buffer b is free once A has read dS of step g - 2 from it
            if (g >= 2 && !mbar_wait(&bar[kLqSFree0 + b], ((g >> 1) - 1) & 1, ctx, 112)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dK = make_sw128_desc(sK0 + (g % SK) * Cfg::kMD, 16, 1024);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
              umma_f16_ss(tmem + Cfg::kColS + 128 * b, desc_advance(dQd, off), desc_advance(dK, off), id_SS,
                          k > 0 ? 1u : 0u);
            }
            umma_commit(&bar[kLqSFull0 + b]);
            if (!mbar_wait(&bar[kLqVFull0 + g % SV], (g / SV) & 1, ctx, 113)) { ok = false; break; }
            // the single dP buffer is free once the epilogue has read dP of step g - 1
            if (g >= 1 && !mbar_wait(&bar[kLqdPRead], (g - 1) & 1, ctx, 114)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dV = make_sw128_desc(sV0 + (g % SV) * Cfg::kMD, 16, 1024);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
              umma_f16_ss(tmem + Cfg::kColdP, desc_advance(ddO, off), desc_advance(dV, off), id_SS,
                          k > 0 ? 1u : 0u);
            }
            umma_commit(&bar[kLqdPFull]);
            umma_commit(&bar[kLqVEmpty0 + g % SV]);
          }
          if (ok) umma_commit(&bar[kLqQEmpty]);
        }
        if (!ok) {
          umma_commit(&bar[kLqDrain]);
          mbar_wait_drain(&bar[kLqDrain], 0, timeout_ns);
        }
      } else {
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
          if (tc > 0 && !mbar_wait(&bar[kLqAccEmpty], (tc - 1) & 1, ctx, 120)) { ok = false; break; }
          for (int j = 0; j < nt; ++j, ++g) {
            const int b = g & 1;
            // dS_j ready (which also orders this after K_j landed: the S MMA
            // that the epilogue waited for read K_j)
            if (!mbar_wait(&bar[kLqEFull0 + b], (g >> 1) & 1, ctx, 121)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dK = make_sw128_desc(sK0 + (g % SK) * Cfg::kMD, kBoxBytes, 1024);
            const uint32_t tS = tmem + Cfg::kColS + 128 * b;
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              umma_f16_ts(tmem + Cfg::kColA, tS + (k >> 2) * 64 + (k & 3) * 8, desc_advance(dK, k * 2048), id_A,
                          (j > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[kLqKEmpty0 + g % SK]);
            umma_commit(&bar[kLqSFree0 + b]);
          }
          if (ok) umma_commit(&bar[kLqAcc]);
        }
        if (!ok) {
          umma_commit(&bar[kLqDrain2]);
          mbar_wait_drain(&bar[kLqDrain2], 0, timeout_ns);
        }
      }
    }
  } else {
    // ---- Epilogue: warp w owns TMEM lane quarter q = w % 4 (query rows
    // 32q..32q+31) and key half c (keys 64c..64c+63 of each key tile).
    const int q = warp & 3;
    const int c = (warp - Cfg::kFirstEpiWarp) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const float sl2 = scale * kLog2e;
    bool ok = true;
    int g = 0, tc = 0;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
      const int h = t / mt;
      const int m = (t - h * mt) * kTile + r;
      // rows past M read 0: their S is 0 (zero-filled Q), so P stays finite
      const float lse2 = m < M ? LSE[static_cast<int64_t>(h) * M + m] * kLog2e : 0.f;
      const float dm = m < M ? Dsum[static_cast<int64_t>(h) * M + m] : 0.f;
      for (int j = 0; j < nt; ++j, ++g) {
        const int b = g & 1;
        if (!mbar_wait(&bar[kLqSFull0 + b], (g >> 1) & 1, ctx, 130)) { ok = false; break; }
        if (!mbar_wait(&bar[kLqdPFull], g & 1, ctx, 131)) { ok = false; break; }
        __syncwarp();
        tc_fence_after();
        uint32_t sa[32], sb[32], da[32], db[32];
        tmem_load_32(lane_base + Cfg::kColdP + 64 * c, da);
        tmem_load_32(lane_base + Cfg::kColdP + 64 * c + 32, db);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[kLqdPRead]);
        tmem_load_32(lane_base + Cfg::kColS + 128 * b + 64 * c, sa);
        tmem_load_32(lane_base + Cfg::kColS + 128 * b + 64 * c + 32, sb);
        uint32_t e[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const uint32_t* sp = x < 16 ? sa + 2 * x : sb + 2 * (x - 16);
          const uint32_t* dp = x < 16 ? da + 2 * x : db + 2 * (x - 16);
          const float p0 = ex2_approx(fmaf(__uint_as_float(sp[0]), sl2, -lse2));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sp[1]), sl2, -lse2));
          e[x] = Elem<T>::pack(p0 * (__uint_as_float(dp[0]) - dm), p1 * (__uint_as_float(dp[1]) - dm));
        }
        tmem_store_32(lane_base + Cfg::kColS + 128 * b + 64 * c, e);
        tmem_store_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[kLqEFull0 + b]);
      }
      if (!ok) break;
      if (!mbar_wait(&bar[kLqAcc], tc & 1, ctx, 132)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      constexpr int kHalf = D / 2;
      // this row's outputs packed to 16-bit as 16-byte chunks, then stored
      // warp-coalesced
      uint4 ch[kHalf / 8];
#pragma unroll
      for (int x = 0; x < kHalf / 32; ++x) {
        uint32_t a[32];
        __syncwarp();  // .sync.aligned TMEM access
        tmem_load_32(lane_base + Cfg::kColA + c * kHalf + 32 * x, a);
#pragma unroll
        for (int y = 0; y < 4; ++y)
          ch[4 * x + y] = make_uint4(
              Elem<T>::pack(scale * __uint_as_float(a[8 * y]), scale * __uint_as_float(a[8 * y + 1])),
              Elem<T>::pack(scale * __uint_as_float(a[8 * y + 2]), scale * __uint_as_float(a[8 * y + 3])),
              Elem<T>::pack(scale * __uint_as_float(a[8 * y + 4]), scale * __uint_as_float(a[8 * y + 5])),
              Elem<T>::pack(scale * __uint_as_float(a[8 * y + 6]), scale * __uint_as_float(a[8 * y + 7])));
      }
      {
        const int row0 = m - lane;  // this warp's first row (query index)
        store_rows_coalesced<kHalf / 8>(
            ch, reinterpret_cast<uint8_t*>(dQ + (static_cast<int64_t>(h) * M + row0) * D + c * kHalf),
            static_cast<size_t>(D) * sizeof(T), lane, M - row0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kLqAccEmpty]);
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

// ============================================================ dkv_lse_kernel
// Persistent, one CTA per SM walking (128-row key tile j, head) items. K_j
// and V_j stay in shared memory; Q_i and dO_i stream (2 slots each). Per
// query tile i, with the key index on the TMEM lanes:
//   S^T  = K_j Q_i^T          (SS, TMEM buffer S)
//   dP^T = V_j dO_i^T         (SS, TMEM buffer X_(g%NX))
//   P^T  = 2^(S^T scale log2e - LSE_i log2e),  dS^T = P^T (dP^T - D_i)
//          (dS warps; both packed to 16-bit into X: dS^T in columns
//          [64c, 64c+32) and P^T in [64c+32, 64c+64) of query half c)
//   dV_j += P^T dO_i,  dK_j += dS^T Q_i   (TS MMAs, A operand from TMEM)
// and finally dK_j = scale dK_j. Columns of queries past M hold finite
// values whose dO and Q rows are zero-filled, so they contribute nothing.
//
// Shared memory (D = 128): K_j 32 KB, V_j 32 KB, Q_i x2, dO_i x2 = 192 KB.
// TMEM: S [0,128), X_b [128 + 128 b, ...), dV and dK after them; NX = 1 for
// D = 128 (512 columns), 2 for D = 64.
// Warps: 0 TMA for K_j, V_j; 1 MMA issuer for S^T and dP^T (TMEM owner);
// 2 TMA for Q_i, dO_i; 3 MMA issuer for dV and dK; 4-11 dS warps.
template <int D>
struct DkvLseCfg {
  static constexpr int kMD = (D / kBoxCols) * kBoxBytes;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kMD;
  static constexpr int kOffQ = 2 * kMD;            // two slots
  static constexpr int kOffdO = kOffQ + 2 * kMD;   // two slots
  static constexpr int kTileBytes = kOffdO + 2 * kMD;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kTileBytes + kBarBytes + 1024;
  static constexpr int kDSWarps = 8;
  static constexpr int kFirstDSWarp = 4;
  static constexpr int kThreads = 32 * (kFirstDSWarp + kDSWarps);
  static constexpr int kNX = D == 128 ? 1 : 2;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColS = 0;
  static constexpr uint32_t kColX = 128;  // + 128 * buffer
  static constexpr uint32_t kColdV = 128 + 128 * kNX;
  static constexpr uint32_t kColdK = kColdV + D;
  static_assert(kColdK + D <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum DkvLseBar : int {
  kLkKV = 0,        // K_j and V_j landed
  kLkKVEmpty = 1,   // the S^T and dP^T MMAs of an item are done with them
  kLkQFull0 = 2,    // + slot
  kLkQEmpty0 = 4,   // + slot: S^T commit + dK commit
  kLkDOFull0 = 6,   // + slot
  kLkDOEmpty0 = 8,  // + slot: dP^T commit + dV commit
  kLkSFull = 10,
  kLkSRead = 11,    // dS warps have read S^T (8 warps)
  kLkXFull0 = 12,   // + X buffer (up to 2)
  kLkEFull0 = 14,   // + X buffer: P^T and dS^T written (8 warps)
  kLkXFree0 = 16,   // + X buffer: dV and dK have read them
  kLkAcc = 18,
  kLkAccEmpty = 19,
  kLkDrain = 20,
  kLkDrain2 = 21,
  kNumDkvLseBars = 22,
};
static_assert(kNumDkvLseBars * 8 + 8 <= 256, "dkv_lse barrier area");

template <typename T, int D>
__global__ void __launch_bounds__(DkvLseCfg<D>::kThreads, 1)
    dkv_lse_kernel(const __grid_constant__ CUtensorMap tm_Q, const __grid_constant__ CUtensorMap tm_K,
                   const __grid_constant__ CUtensorMap tm_V, const __grid_constant__ CUtensorMap tm_dO,
                   const float* __restrict__ LSE, const float* __restrict__ Dsum, T* __restrict__ dK,
                   T* __restrict__ dV, int M, int N, int H, float scale, KernelStatus* status,
                   uint64_t timeout_ns) {
  using Cfg = DkvLseCfg<D>;
  constexpr int NX = Cfg::kNX;
  constexpr int kEpi = Cfg::kDSWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumDkvLseBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int mt = (M + kTile - 1) / kTile;
  const int ntk = (N + kTile - 1) / kTile;
  const int tiles = ntk * H;

  if (threadIdx.x == 0) {
    mbar_init(&bar[kLkKV], 1);
    mbar_init(&bar[kLkKVEmpty], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[kLkQFull0 + s], 1);
      mbar_init(&bar[kLkQEmpty0 + s], 2);
      mbar_init(&bar[kLkDOFull0 + s], 1);
      mbar_init(&bar[kLkDOEmpty0 + s], 2);
    }
    mbar_init(&bar[kLkSFull], 1);
    mbar_init(&bar[kLkSRead], kEpi);
    for (int b = 0; b < NX; ++b) {
      mbar_init(&bar[kLkXFull0 + b], 1);
      mbar_init(&bar[kLkEFull0 + b], kEpi);
      mbar_init(&bar[kLkXFree0 + b], 1);
    }
    mbar_init(&bar[kLkAcc], 1);
    mbar_init(&bar[kLkAccEmpty], kEpi);
    mbar_init(&bar[kLkDrain], 1);
    mbar_init(&bar[kLkDrain2], 1);
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
    // ---- TMA producer for the resident K_j and V_j of each item
    if (lane == 0) {
      tma_prefetch_desc(&tm_K);
      tma_prefetch_desc(&tm_V);
      const uint64_t pol = l2_policy_evict_normal();
      int nkv = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int h = t / ntk;
        const int n0 = (t - h * ntk) * kTile;
        if (nkv > 0 && !mbar_wait(&bar[kLkKVEmpty], (nkv - 1) & 1, ctx, 140)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar[kLkKV], 2 * Cfg::kMD);
#pragma unroll
        for (int b = 0; b < D / kBoxCols; ++b) {
          tma_load_3d(smem + Cfg::kOffK + b * kBoxBytes, &tm_K, &bar[kLkKV], b * kBoxCols, n0, h, pol);
          tma_load_3d(smem + Cfg::kOffV + b * kBoxBytes, &tm_V, &bar[kLkKV], b * kBoxCols, n0, h, pol);
        }
        ++nkv;
      }
      if (*abort_flag && nkv > 0) mbar_wait_drain(&bar[kLkKV], (nkv - 1) & 1, timeout_ns);
    }
  } else if (warp == 2) {
    // ---- TMA producer for the streamed Q_i and dO_i (two slots each; every
    // key-tile CTA of the head reads them, so they are L2 hits for all but
    // the first). Polls both "empty" barriers without blocking and issues
    // whichever load can go. No L2 prefetch ahead: it shares the TMA unit
    // and L2 queues with the loads and cost 3 % of the call here.
    if (lane == 0) {
      tma_prefetch_desc(&tm_dO);
      tma_prefetch_desc(&tm_Q);
      const uint64_t pol = l2_policy_evict_last();
      const int my_items = (tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                           static_cast<int>(gridDim.x);
      const int total = my_items * mt;
      auto head_of = [&](int g) { return (static_cast<int>(blockIdx.x) + (g / mt) * static_cast<int>(gridDim.x)) / ntk; };
      int next_do = 0, next_q = 0;
      uint64_t t_last = global_timer_ns();
      bool failed = false;
      while ((next_do < total || next_q < total) && !failed) {
        bool progressed = false;
        if (next_q < total && (next_q < 2 || mbar_poll(&bar[kLkQEmpty0 + (next_q & 1)], ((next_q >> 1) - 1) & 1))) {
          const int s = next_q & 1;
          const int hh = head_of(next_q), i = next_q % mt;
          mbar_arrive_expect_tx(&bar[kLkQFull0 + s], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffQ + s * Cfg::kMD + b * kBoxBytes, &tm_Q, &bar[kLkQFull0 + s],
                        b * kBoxCols, i * kTile, hh, pol);
          ++next_q;
          progressed = true;
        }
        if (next_do < total && (next_do < 2 || mbar_poll(&bar[kLkDOEmpty0 + (next_do & 1)], ((next_do >> 1) - 1) & 1))) {
          const int s = next_do & 1;
          const int hh = head_of(next_do), i = next_do % mt;
          mbar_arrive_expect_tx(&bar[kLkDOFull0 + s], Cfg::kMD);
#pragma unroll
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d(smem + Cfg::kOffdO + s * Cfg::kMD + b * kBoxBytes, &tm_dO, &bar[kLkDOFull0 + s],
                        b * kBoxCols, i * kTile, hh, pol);
          ++next_do;
          progressed = true;
        }
        if (progressed) {
          t_last = global_timer_ns();
        } else {
          if (*abort_flag) break;
          if (global_timer_ns() - t_last > timeout_ns) {
            note_failure(ctx, 141);
            failed = true;
          }
        }
      }
      if (*abort_flag) {
        for (int i = (next_do > 2 ? next_do - 2 : 0); i < next_do; ++i)
          mbar_wait_drain(&bar[kLkDOFull0 + (i & 1)], (i >> 1) & 1, timeout_ns);
        for (int i = (next_q > 2 ? next_q - 2 : 0); i < next_q; ++i)
          mbar_wait_drain(&bar[kLkQFull0 + (i & 1)], (i >> 1) & 1, timeout_ns);
      }
    }
  } else if (warp == 1 || warp == 3) {
    if (lane == 0) {
      constexpr bool kB = Elem<T>::kBF16;
      // S^T = K_j Q_i^T, dP^T = V_j dO_i^T: A and B K-major over d
      constexpr uint32_t id_SS = make_idesc_f16<kB>(kTile, kTile, false, false);
      // dV += P^T dO_i, dK += dS^T Q_i: A from TMEM, B MN-major (N = d)
      constexpr uint32_t id_TS = make_idesc_f16<kB>(kTile, D, false, true);
      const uint64_t dKt = make_sw128_desc(smem_u32(smem + Cfg::kOffK), 16, 1024);
      const uint64_t dVt = make_sw128_desc(smem_u32(smem + Cfg::kOffV), 16, 1024);
      bool ok = true;
      if (warp == 1) {
        int g = 0, tc = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
          if (!mbar_wait(&bar[kLkKV], tc & 1, ctx, 150)) { ok = false; break; }
          for (int i = 0; i < mt; ++i, ++g) {
            const int s = g & 1;
            const int xb = g % NX;
            if (!mbar_wait(&bar[kLkQFull0 + s], (g >> 1) & 1, ctx, 151)) { ok = false; break; }
            if (g >= 1 && !mbar_wait(&bar[kLkSRead], (g - 1) & 1, ctx, 152)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dQs = make_sw128_desc(smem_u32(smem + Cfg::kOffQ + s * Cfg::kMD), 16, 1024);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
              umma_f16_ss(tmem + Cfg::kColS, desc_advance(dKt, off), desc_advance(dQs, off), id_SS,
                          k > 0 ? 1u : 0u);
            }
            umma_commit(&bar[kLkSFull]);
            umma_commit(&bar[kLkQEmpty0 + s]);
            if (!mbar_wait(&bar[kLkDOFull0 + s], (g >> 1) & 1, ctx, 153)) { ok = false; break; }
            // X buffer xb is free once dV and dK of step g - NX have read it
            if (g >= NX && !mbar_wait(&bar[kLkXFree0 + xb], ((g / NX) - 1) & 1, ctx, 154)) { ok = false; break; }
            tc_fence_after();
            const uint64_t ddO = make_sw128_desc(smem_u32(smem + Cfg::kOffdO + s * Cfg::kMD), 16, 1024);
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t off = (k >> 2) * kBoxBytes + (k & 3) * 32;
              umma_f16_ss(tmem + Cfg::kColX + 128 * xb, desc_advance(dVt, off), desc_advance(ddO, off), id_SS,
                          k > 0 ? 1u : 0u);
            }
            umma_commit(&bar[kLkXFull0 + xb]);
            umma_commit(&bar[kLkDOEmpty0 + s]);
          }
          if (ok) umma_commit(&bar[kLkKVEmpty]);
        }
        if (!ok) {
          umma_commit(&bar[kLkDrain]);
          mbar_wait_drain(&bar[kLkDrain], 0, timeout_ns);
        }
      } else {
        int g = 0, tc = 0;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
          if (tc > 0 && !mbar_wait(&bar[kLkAccEmpty], (tc - 1) & 1, ctx, 160)) { ok = false; break; }
          for (int i = 0; i < mt; ++i, ++g) {
            const int s = g & 1;
            const int xb = g % NX;
            // P^T and dS^T ready (after the S^T / dP^T MMAs that read Q_i and
            // dO_i, so those slots have landed too)
            if (!mbar_wait(&bar[kLkEFull0 + xb], (g / NX) & 1, ctx, 161)) { ok = false; break; }
            tc_fence_after();
            const uint32_t tX = tmem + Cfg::kColX + 128 * xb;
            const uint64_t ddO = make_sw128_desc(smem_u32(smem + Cfg::kOffdO + s * Cfg::kMD), kBoxBytes, 1024);
            const uint64_t dQs = make_sw128_desc(smem_u32(smem + Cfg::kOffQ + s * Cfg::kMD), kBoxBytes, 1024);
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              // P^T for queries 16k..16k+15: query half k >> 2, packed columns
              // 32..63 of that half, 8 per step
              umma_f16_ts(tmem + Cfg::kColdV, tX + (k >> 2) * 64 + 32 + (k & 3) * 8, desc_advance(ddO, k * 2048),
                          id_TS, (i > 0 || k > 0) ? 1u : 0u);
            }
#pragma unroll
            for (int k = 0; k < kTile / 16; ++k) {
              umma_f16_ts(tmem + Cfg::kColdK, tX + (k >> 2) * 64 + (k & 3) * 8, desc_advance(dQs, k * 2048), id_TS,
                          (i > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[kLkDOEmpty0 + s]);
            umma_commit(&bar[kLkQEmpty0 + s]);
            umma_commit(&bar[kLkXFree0 + xb]);
          }
          if (ok) umma_commit(&bar[kLkAcc]);
        }
        if (!ok) {
          umma_commit(&bar[kLkDrain2]);
          mbar_wait_drain(&bar[kLkDrain2], 0, timeout_ns);
        }
      }
    }
  } else if (warp >= Cfg::kFirstDSWarp) {
    // ---- dS warps: lane quarter qq = warp % 4 (keys 32qq..32qq+31 as two
    // 16-lane halves), query half c. In the .16x256b fragment thread t holds
    // keys t/4 and 8 + t/4 of a half and queries 8 blk + 2 (t%4) + {0,1}.
    const int qq = warp & 3;
    const int c = (warp - Cfg::kFirstDSWarp) >> 2;
    const int lq = lane & 3;
    const float sl2 = scale * kLog2e;
    bool ok = true;
    int g = 0, tc = 0;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
      const int h = t / ntk;
      const int n0 = (t - h * ntk) * kTile;
      for (int i = 0; i < mt; ++i, ++g) {
        const int xb = g % NX;
        // LSE (log2 units) and D for this thread's 16 queries; queries past M read 0
        float L2[16], Dv[16];
        {
          const int64_t row0 = static_cast<int64_t>(h) * M;
          const int q0 = i * kTile + 64 * c + 2 * lq;
#pragma unroll
          for (int blk = 0; blk < 8; ++blk) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int qi = q0 + 8 * blk + u;
              L2[2 * blk + u] = qi < M ? __ldg(LSE + row0 + qi) * kLog2e : 0.f;
              Dv[2 * blk + u] = qi < M ? __ldg(Dsum + row0 + qi) : 0.f;
            }
          }
        }
        if (!mbar_wait(&bar[kLkSFull], g & 1, ctx, 170)) { ok = false; break; }
        __syncwarp();
        tc_fence_after();
        uint32_t s0[32], s1[32];
        tmem_load_16x256b_x8(tmem + Cfg::kColS + 64 * c + (static_cast<uint32_t>(32 * qq) << 16), s0);
        tmem_load_16x256b_x8(tmem + Cfg::kColS + 64 * c + (static_cast<uint32_t>(32 * qq + 16) << 16), s1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[kLkSRead]);
        if (!mbar_wait(&bar[kLkXFull0 + xb], (g / NX) & 1, ctx, 171)) { ok = false; break; }
        __syncwarp();
        tc_fence_after();
        const uint32_t tX = tmem + Cfg::kColX + 128 * xb + 64 * c;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t lane_addr = static_cast<uint32_t>(32 * qq + 16 * hh) << 16;
          uint32_t dp[32];
          tmem_load_16x256b_x8(tX + lane_addr, dp);
          const uint32_t* sv = hh == 0 ? s0 : s1;
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int blk = 0; blk < 8; ++blk) {
            float p[4], ds[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int qv = 2 * blk + (u & 1);
              p[u] = ex2_approx(fmaf(__uint_as_float(sv[4 * blk + u]), sl2, -L2[qv]));
              ds[u] = p[u] * (__uint_as_float(dp[4 * blk + u]) - Dv[qv]);
            }
            pk[2 * blk] = Elem<T>::pack(p[0], p[1]);
            pk[2 * blk + 1] = Elem<T>::pack(p[2], p[3]);
            dk[2 * blk] = Elem<T>::pack(ds[0], ds[1]);
            dk[2 * blk + 1] = Elem<T>::pack(ds[2], ds[3]);
          }
          tmem_store_16x128b_x8(tX + lane_addr, dk);
          tmem_store_16x128b_x8(tX + 32 + lane_addr, pk);
        }
        tmem_store_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[kLkEFull0 + xb]);
      }
      if (!ok) break;
      // final dV_j and dK_j rows (lane = key) -> 16-bit outputs
      if (!mbar_wait(&bar[kLkAcc], tc & 1, ctx, 172)) { ok = false; break; }
      __syncwarp();
      tc_fence_after();
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(qq * 32) << 16);
      constexpr int kHalf = D / 2;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = (which == 0 ? Cfg::kColdV : Cfg::kColdK) + c * kHalf;
        const float mul = which == 0 ? 1.f : scale;
        uint4 ch[kHalf / 8];  // this row, packed to 16-bit, stored warp-coalesced
#pragma unroll
        for (int x = 0; x < kHalf / 32; ++x) {
          uint32_t v[32];
          __syncwarp();  // .sync.aligned TMEM access: the warp reconverges after the
                         // row-guarded stores of the previous iteration
          tmem_load_32(lane_base + col + x * 32, v);
#pragma unroll
          for (int y = 0; y < 4; ++y)
            ch[4 * x + y] = make_uint4(
                Elem<T>::pack(mul * __uint_as_float(v[8 * y]), mul * __uint_as_float(v[8 * y + 1])),
                Elem<T>::pack(mul * __uint_as_float(v[8 * y + 2]), mul * __uint_as_float(v[8 * y + 3])),
                Elem<T>::pack(mul * __uint_as_float(v[8 * y + 4]), mul * __uint_as_float(v[8 * y + 5])),
                Elem<T>::pack(mul * __uint_as_float(v[8 * y + 6]), mul * __uint_as_float(v[8 * y + 7])));
        }
        __syncwarp();
        const int row0 = n0 + qq * 32;  // this warp's first row (key index)
        store_rows_coalesced<kHalf / 8>(
            ch,
            reinterpret_cast<uint8_t*>((which == 0 ? dV : dK) + (static_cast<int64_t>(h) * N + row0) * D +
                                       c * kHalf),
            static_cast<size_t>(D) * sizeof(T), lane, N - row0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kLkAccEmpty]);
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

// ================================================================ host side
template <typename T>
void set_lse_attrs() {
  cudaFuncSetAttribute(dq_lse_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize, DqLseCfg<128>::kSmemBytes);
  cudaFuncSetAttribute(dq_lse_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, DqLseCfg<64>::kSmemBytes);
  cudaFuncSetAttribute(dkv_lse_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DkvLseCfg<128>::kSmemBytes);
  cudaFuncSetAttribute(dkv_lse_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DkvLseCfg<64>::kSmemBytes);
}

// Checks, D workspace, tensor maps and the three launches on `stream`
// (stream-ordered; in-kernel wait timeouts are read with
// fmha_bwd_poll_device_status after the stream finished).
template <typename T>
int run_backward_lse(T* dQ, T* dK, T* dV, const T* Q, const T* K, const T* V, const T* O, const T* dO,
                     const float* LSE, int M, int N, int D, int H, float scale, cudaStream_t stream) {
  int rc = check_args(dQ, dK, dV, Q, K, V, /*P=*/O, dO, M, N, D, H, /*p_rows=*/false);
  if (rc != kOk) return rc;
  if (static_cast<int64_t>(H) * M / 16 + 1 > 0x7fffffffLL)
    return set_error(kErrInvalidArgument, "total_heads * M too large");
  if (!LSE) return set_error(kErrInvalidArgument, "null LSE argument");
  if ((reinterpret_cast<uintptr_t>(LSE) & 3u) != 0) return set_error(kErrMisaligned, "LSE must be 4-byte aligned");
  if (!(scale > 0.f) || !(scale < 3.0e38f))
    return set_error(kErrInvalidArgument, "softmax_scale must be positive and finite");
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kErrLaunch, "no current CUDA device");
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0)
    return set_error(kErrUnsupportedDevice, "device %d is sm_%d%d; this library needs sm_100", device, major, minor);
  const size_t rows = static_cast<size_t>(H) * static_cast<size_t>(M);
  DeviceWorkspace* w = get_workspace<T>(device, rows);
  if (!w) return kErrOutOfMemory;
  {
    static std::once_flag once[64];
    if (device < 64) std::call_once(once[device], [] { set_lse_attrs<T>(); });
    else set_lse_attrs<T>();
  }
  if (!encode_fn()) return set_error(kErrNoDriver, "cuTensorMapEncodeTiled is unavailable");
  constexpr bool kBF16 = Elem<T>::kBF16;
  CUtensorMap mQ, mK, mV, mdO;
  if (!encode_map(&mQ, kBF16, Q, D, M, H) || !encode_map(&mK, kBF16, K, D, N, H) ||
      !encode_map(&mV, kBF16, V, D, N, H) || !encode_map(&mdO, kBF16, dO, D, M, H))
    return set_error(kErrInvalidArgument, "tensor map encoding failed (M=%d N=%d K_dim=%d heads=%d)", M, N, D, H);
  const uint64_t tmo = effective_timeout_ns();
  const int sms = w->sm_count > 0 ? w->sm_count : 148;
  const long long qitems = static_cast<long long>((M + kTile - 1) / kTile) * H;
  const long long kitems = static_cast<long long>((N + kTile - 1) / kTile) * H;
  const dim3 grid_rows(static_cast<unsigned>(qitems < sms ? qitems : sms));
  const dim3 grid_cols(static_cast<unsigned>(kitems < sms ? kitems : sms));
  const int64_t nrows = static_cast<int64_t>(rows);
  float* dsum = w->dsum;
  KernelStatus* st = w->host_status_dev;
  if (D == 128) {
    const unsigned blocks = static_cast<unsigned>((nrows + 15) / 16);
    rowsum_do_o_kernel<T, 128><<<blocks, 256, 0, stream>>>(dO, O, dsum, nrows);
    dq_lse_kernel<T, 128><<<grid_rows, DqLseCfg<128>::kThreads, DqLseCfg<128>::kSmemBytes, stream>>>(
        mQ, mK, mV, mdO, LSE, dsum, dQ, M, N, H, scale, st, tmo);
    dkv_lse_kernel<T, 128><<<grid_cols, DkvLseCfg<128>::kThreads, DkvLseCfg<128>::kSmemBytes, stream>>>(
        mQ, mK, mV, mdO, LSE, dsum, dK, dV, M, N, H, scale, st, tmo);
  } else {
    const unsigned blocks = static_cast<unsigned>((nrows + 31) / 32);
    rowsum_do_o_kernel<T, 64><<<blocks, 256, 0, stream>>>(dO, O, dsum, nrows);
    dq_lse_kernel<T, 64><<<grid_rows, DqLseCfg<64>::kThreads, DqLseCfg<64>::kSmemBytes, stream>>>(
        mQ, mK, mV, mdO, LSE, dsum, dQ, M, N, H, scale, st, tmo);
    dkv_lse_kernel<T, 64><<<grid_cols, DkvLseCfg<64>::kThreads, DkvLseCfg<64>::kSmemBytes, stream>>>(
        mQ, mK, mV, mdO, LSE, dsum, dK, dV, M, N, H, scale, st, tmo);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kErrLaunch, "launch failed: %s", cudaGetErrorString(e));
  return set_error(kOk, "");
}

}  // namespace fmha_sm100
