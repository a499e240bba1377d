// CPU oracle for the attention-backward path. TEST INFRASTRUCTURE ONLY.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
// load this library, and only as the checker; the product path (the CUDA
// libraries under build/) never links or calls it.
//
// This is a restatement of the reference's CPU algorithm,
// src/kernel/correct/cpu_reference.hpp:74-126 (fmha_backward_cpu) with
// softmax_backward at :30-40, generalised over the input storage type
// (bf16 or fp16 bits) and over heads:
//
//   dP[m,n] = sum_k dO[m,k] * V[n,k]                  (fp32, :79-88)
//   D[m]    = sum_n dP[m,n] * P[m,n]                  (fp32 rowsum, :32-35)
//   dS[m,n] = P[m,n] * (dP[m,n] - D[m])               (fp32, :36-38)
//   dQ[m,k] = sum_n dS[m,n] * K[n,k]                  (:95-103)
//   dK[n,k] = sum_m dS[m,n] * Q[m,k]                  (:106-114)
//   dV[n,k] = sum_m P[m,n]  * dO[m,k]                 (:117-125)
//
// No softmax scale is applied anywhere (the reference applies none in the
// backward pass). P is consumed as fp32 upcast from its storage type, as the
// reference's `const float* P` argument implies (:75). Outputs are returned in
// fp32 (before the reference's final half_cast) so tests can measure the
// error of the 16-bit GPU outputs against the unrounded result.
//
// Per-head layout (row-major, heads contiguous), matching the C-ABI in
// src/fmha_bwd_kernels.hip:475-477: Q/dO/dQ at h*M*d, K/V/dK/dV at h*N*d,
// P at h*M*N. All offsets are 64-bit.
//
// The dK/dV loops are reordered (m outer, n/k inner) so the oracle walks
// memory contiguously; every sum is still a plain fp32 accumulation over the
// same terms, so it agrees with the reference to fp32 rounding.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline float bf16_to_f32(uint16_t b) {
  uint32_t u = static_cast<uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline float fp16_to_f32(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return static_cast<float>(v);
}

using Decode = float (*)(uint16_t);

// One head of the backward pass; all inputs already decoded to fp32.
void backward_one_head(const float* Q, const float* K, const float* V,
                       const float* P, const float* dO, float* dQ, float* dK,
                       float* dV, float* Dsum, int64_t M, int64_t N,
                       int64_t d) {
  std::vector<float> dS(static_cast<size_t>(M * N));
  // dP and softmax backward (cpu_reference.hpp:79-92, :30-40)
  std::vector<float> dProw(static_cast<size_t>(N));
  for (int64_t m = 0; m < M; ++m) {
    const float* dOm = dO + m * d;
    for (int64_t n = 0; n < N; ++n) {
      const float* Vn = V + n * d;
      float s = 0.0f;
      for (int64_t k = 0; k < d; ++k) s += dOm[k] * Vn[k];
      dProw[n] = s;
    }
    const float* Pm = P + m * N;
    float rowsum = 0.0f;
    for (int64_t n = 0; n < N; ++n) rowsum += dProw[n] * Pm[n];
    if (Dsum) Dsum[m] = rowsum;
    float* dSm = dS.data() + m * N;
    for (int64_t n = 0; n < N; ++n) dSm[n] = Pm[n] * (dProw[n] - rowsum);
  }
  // dQ = dS K (cpu_reference.hpp:95-103)
  for (int64_t m = 0; m < M; ++m) {
    float* dQm = dQ + m * d;
    for (int64_t k = 0; k < d; ++k) dQm[k] = 0.0f;
    const float* dSm = dS.data() + m * N;
    for (int64_t n = 0; n < N; ++n) {
      const float s = dSm[n];
      const float* Kn = K + n * d;
      for (int64_t k = 0; k < d; ++k) dQm[k] += s * Kn[k];
    }
  }
  // dK = dS^T Q and dV = P^T dO (cpu_reference.hpp:106-125)
  std::memset(dK, 0, sizeof(float) * static_cast<size_t>(N * d));
  std::memset(dV, 0, sizeof(float) * static_cast<size_t>(N * d));
  for (int64_t m = 0; m < M; ++m) {
    const float* Qm = Q + m * d;
    const float* dOm = dO + m * d;
    const float* dSm = dS.data() + m * N;
    const float* Pm = P + m * N;
    for (int64_t n = 0; n < N; ++n) {
      const float s = dSm[n];
      const float p = Pm[n];
      float* dKn = dK + n * d;
      float* dVn = dV + n * d;
      for (int64_t k = 0; k < d; ++k) {
        dKn[k] += s * Qm[k];
        dVn[k] += p * dOm[k];
      }
    }
  }
}

void decode(const uint16_t* src, float* dst, int64_t count, Decode f) {
  for (int64_t i = 0; i < count; ++i) dst[i] = f(src[i]);
}

int run(const uint16_t* Q, const uint16_t* K, const uint16_t* V,
        const uint16_t* P, const uint16_t* dO, float* dQ, float* dK,
        float* dV, float* Dsum, int M, int N, int d, int H, int threads,
        Decode f) {
  if (M <= 0 || N <= 0 || d <= 0 || H <= 0) return 1;
  if (threads < 1) threads = 1;
  const int64_t Mq = M, Nq = N, dq = d;
  auto worker = [&](int h) {
    const int64_t hq = h;
    std::vector<float> q(Mq * dq), k(Nq * dq), v(Nq * dq), p(Mq * Nq),
        o(Mq * dq);
    decode(Q + hq * Mq * dq, q.data(), Mq * dq, f);
    decode(K + hq * Nq * dq, k.data(), Nq * dq, f);
    decode(V + hq * Nq * dq, v.data(), Nq * dq, f);
    decode(P + hq * Mq * Nq, p.data(), Mq * Nq, f);
    decode(dO + hq * Mq * dq, o.data(), Mq * dq, f);
    backward_one_head(q.data(), k.data(), v.data(), p.data(), o.data(),
                      dQ + hq * Mq * dq, dK + hq * Nq * dq, dV + hq * Nq * dq,
                      Dsum ? Dsum + hq * Mq : nullptr, Mq, Nq, dq);
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t]() {
      for (int h = t; h < H; h += threads) worker(h);
    });
  }
  for (auto& th : pool) th.join();
  return 0;
}

}  // namespace

extern "C" {

// Inputs are raw 16-bit storage (bf16 or fp16 bits); outputs are fp32.
// Dsum (optional, may be null) receives the per-row rowsum D[h*M + m].
// Returns 0 on success, 1 on invalid sizes.
int oracle_fmha_bwd_bf16(const uint16_t* Q, const uint16_t* K,
                         const uint16_t* V, const uint16_t* P,
                         const uint16_t* dO, float* dQ, float* dK, float* dV,
                         float* Dsum, int M, int N, int d, int H,
                         int threads) {
  return run(Q, K, V, P, dO, dQ, dK, dV, Dsum, M, N, d, H, threads,
             bf16_to_f32);
}

int oracle_fmha_bwd_fp16(const uint16_t* Q, const uint16_t* K,
                         const uint16_t* V, const uint16_t* P,
                         const uint16_t* dO, float* dQ, float* dK, float* dV,
                         float* Dsum, int M, int N, int d, int H,
                         int threads) {
  return run(Q, K, V, P, dO, dQ, dK, dV, Dsum, M, N, d, H, threads,
             fp16_to_f32);
}

}  // extern "C"
