// Host side of the attention-backward C-ABI: argument checks, per-device
// workspace, TMA tensor maps and the two launches. Included once by each
// library translation unit (bf16 and fp16), which instantiates it for its
// element type and defines the extern "C" entry points.
//
// Replaces the body of fmha_bwd_full_py (src/fmha_bwd_kernels.hip:475-523)
// and fmha_bwd_full_fp16 (src/fmha_bwd_kernels_fp16.hip:236-280):
//   * no per-call dP/dS allocation (those never leave the SM); the only
//     workspace is the H*M fp32 rowsum D, cached per device and grown on
//     demand;
//   * shapes and pointers are checked before anything is launched, so a bad
//     call leaves the outputs untouched and reports an error code;
//   * 64-bit offsets throughout.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>

#include "fmha_bwd_kernels.cuh"

namespace fmha_sm100 {

// Error codes returned by the entry points and by fmha_bwd_last_error().
enum FmhaError : int {
  kOk = 0,
  kErrInvalidArgument = 1,   // null pointer, non-positive or unsupported size
  kErrMisaligned = 2,        // pointer or row pitch not 16-byte aligned
  kErrUnsupportedDevice = 3, // not an sm_100 device
  kErrOutOfMemory = 4,       // workspace allocation failed
  kErrLaunch = 5,            // CUDA launch or runtime error
  kErrDeviceTimeout = 6,     // an in-kernel wait ran out of time (see status)
  kErrNoDriver = 7,          // cuTensorMapEncodeTiled unavailable
};

struct ErrorState {
  std::atomic<int> code{0};
  std::mutex mu;
  char message[512] = {0};
};

inline ErrorState& error_state() {
  static ErrorState s;
  return s;
}

inline int set_error(int code, const char* fmt, ...) {
  ErrorState& s = error_state();
  std::lock_guard<std::mutex> g(s.mu);
  s.code.store(code);
  if (code == kOk) {
    s.message[0] = 0;
    return code;
  }
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(s.message, sizeof(s.message), fmt, ap);
  va_end(ap);
  fprintf(stderr, "fmha_bwd: %s\n", s.message);
  return code;
}

// ---------------------------------------------------------------- driver
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D map over a [heads][rows][cols] row-major 16-bit tensor, box of
// 64 columns x `box_rows` rows x 1 head, 128-byte swizzle, zero fill out of
// bounds.
inline bool encode_map(CUtensorMap* map, bool bf16, const void* base, uint64_t cols,
                       uint64_t rows, uint64_t heads, uint32_t box_rows = kTile) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {cols, rows, heads};
  const cuuint64_t strides[2] = {cols * 2, rows * cols * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBoxCols), box_rows, 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------- workspace
struct DeviceWorkspace {
  float* dsum = nullptr;
  size_t dsum_floats = 0;
  float* part = nullptr;     // fp32 partials of split tail items
  size_t part_floats = 0;
  KernelStatus* host_status = nullptr;      // mapped pinned host memory
  KernelStatus* host_status_dev = nullptr;  // its device address
  bool attrs_set = false;
  int sm_count = 0;
};

inline std::mutex& ws_mutex() {
  static std::mutex m;
  return m;
}
inline std::map<int, DeviceWorkspace>& ws_map() {
  static std::map<int, DeviceWorkspace> m;
  return m;
}

inline uint64_t wait_timeout_ns() {
  static std::atomic<uint64_t> cached{0};
  uint64_t v = cached.load();
  if (v == 0) {
    uint64_t ms = 4000;
    if (const char* e = getenv("FMHA_BWD_WAIT_TIMEOUT_MS")) {
      long long x = atoll(e);
      if (x > 0) ms = static_cast<uint64_t>(x);
    }
    v = ms * 1000000ull;
    cached.store(v);
  }
  return v;
}

inline std::atomic<uint64_t>& timeout_override_ns() {
  static std::atomic<uint64_t> v{0};
  return v;
}

inline uint64_t effective_timeout_ns() {
  uint64_t o = timeout_override_ns().load();
  return o ? o : wait_timeout_ns();
}

template <typename T>
void set_kernel_attrs() {
  cudaFuncSetAttribute(dq_kernel<T, 64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DqCfg<64>::kSmemBytes);
  cudaFuncSetAttribute(dq_kernel<T, 128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DqCfg<128>::kSmemBytes);
  cudaFuncSetAttribute(dq_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DqCfg<64>::kSmemBytes);
  cudaFuncSetAttribute(dq_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DqCfg<128>::kSmemBytes);
  cudaFuncSetAttribute(dkv_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DkvCfg<64>::kSmemBytes);
  cudaFuncSetAttribute(dkv_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       DkvCfg<128>::kSmemBytes);
}

// The status slot of `device`, allocated on first use (caller holds
// ws_mutex). Returns false (error recorded) if the allocation fails.
inline bool ensure_status_slot(int device, DeviceWorkspace& w) {
  if (!w.host_status) {
    if (cudaHostAlloc(&w.host_status, sizeof(KernelStatus),
                      cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
        cudaHostGetDevicePointer(&w.host_status_dev, w.host_status, 0) != cudaSuccess) {
      set_error(kErrOutOfMemory, "host status slot allocation failed");
      return false;
    }
    memset(w.host_status, 0, sizeof(KernelStatus));
    cudaDeviceGetAttribute(&w.sm_count, cudaDevAttrMultiProcessorCount, device);
  }
  return true;
}

// Work units for `items` items of `len` steps each on `grid` CTAs. The
// items fill `items / grid` whole waves; the `tail` left over would run as
// one partly filled wave. Splitting each tail item into q parts (q <= 4,
// parts of at least 8 steps) runs the tail as ceil(q tail / grid) waves of
// parts 1/q as long, so the tail costs ceil(q tail / grid) / q item times
// instead of one; the q with the lowest cost is taken when it saves at least
// a tenth of an item time (a part carries fixed costs: its first operand
// tiles, the readout of fp32 partials, a share of the combine kernel).
// Items shorter than kMinSplitLen steps stay whole. Examples on 148 CTAs:
// 192 items (a tail of 44) -> 3 parts, one wave of parts, 1/3 of an item
// time; 1280 items (tail 96) -> 3 parts, two waves of parts, 2/3; 864 items
// (tail 124) -> no split. Splitting needs a partial-sum workspace; without
// one (`allow` false) every item stays whole.
constexpr int kMinSplitLen = 16;
inline UnitMap plan_units(int items, int grid, int len, bool allow) {
  UnitMap um{items, 1, items};
  if (!allow || grid <= 0 || len < kMinSplitLen) return um;
  const int waves = items / grid, tail = items - waves * grid;
  if (tail == 0) return um;
  int best_q = 1;
  double best = 1.0;
  for (int q = 2; q <= kMaxParts && len / q >= 8; ++q) {
    const double cost = static_cast<double>((q * tail + grid - 1) / grid) / q;
    if (cost < best - 0.1) {
      best = cost;
      best_q = q;
    }
  }
  if (best_q == 1) return um;
  um.full = waves * grid;
  um.parts = best_q;
  um.units = um.full + best_q * tail;
  return um;
}

// Returns the workspace of the current device with at least the requested
// capacity, or nullptr (error already recorded).
template <typename T>
DeviceWorkspace* get_workspace(int device, size_t dsum_floats, size_t part_floats = 0) {
  std::lock_guard<std::mutex> g(ws_mutex());
  DeviceWorkspace& w = ws_map()[device];
  if (!ensure_status_slot(device, w)) return nullptr;
  if (!w.attrs_set) {
    set_kernel_attrs<T>();
    w.attrs_set = true;
  }
  if (dsum_floats > w.dsum_floats) {
    if (w.dsum) cudaFree(w.dsum);
    w.dsum = nullptr;
    w.dsum_floats = 0;
    if (cudaMalloc(&w.dsum, dsum_floats * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      set_error(kErrOutOfMemory, "workspace allocation of %zu bytes failed",
                dsum_floats * sizeof(float));
      return nullptr;
    }
    w.dsum_floats = dsum_floats;
  }
  if (part_floats > w.part_floats) {
    if (w.part) cudaFree(w.part);
    w.part = nullptr;
    w.part_floats = 0;
    if (cudaMalloc(&w.part, part_floats * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      w.part = nullptr;
      set_error(kErrOutOfMemory, "workspace allocation of %zu bytes failed",
                part_floats * sizeof(float));
      return nullptr;
    }
    w.part_floats = part_floats;
  }
  return &w;
}

// Field-wise volatile read of a status slot written by the device.
inline KernelStatus read_status(const KernelStatus* p) {
  const volatile int* v = reinterpret_cast<const volatile int*>(p);
  KernelStatus s;
  s.code = v[0];
  s.where = v[1];
  s.block = v[2];
  s.pad = 0;
  return s;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Validates the call. Returns kOk or an error code (already recorded).
// `p_rows`: the call reads an [M][N] 16-bit P, whose rows must start on
// 16-byte boundaries (N % 8 == 0); the recompute-P entries pass false.
inline int check_args(const void* dQ, const void* dK, const void* dV, const void* Q,
                      const void* K, const void* V, const void* P, const void* dO, int M,
                      int N, int D, int H, bool p_rows = true) {
  if (!dQ || !dK || !dV || !Q || !K || !V || !P || !dO)
    return set_error(kErrInvalidArgument, "null pointer argument");
  if (M <= 0 || N <= 0 || H <= 0 || D <= 0)
    return set_error(kErrInvalidArgument, "sizes must be positive (M=%d N=%d K_dim=%d heads=%d)", M,
                     N, D, H);
  if (D != 64 && D != 128)
    return set_error(kErrInvalidArgument, "K_dim=%d unsupported (64 or 128)", D);
  if (H > 65535) return set_error(kErrInvalidArgument, "total_heads=%d exceeds 65535", H);
  if (p_rows && N % 8 != 0)
    return set_error(kErrMisaligned, "N=%d: P rows must be a multiple of 16 bytes (N %% 8 == 0)", N);
  if (!aligned16(dQ) || !aligned16(dK) || !aligned16(dV) || !aligned16(Q) || !aligned16(K) ||
      !aligned16(V) || !aligned16(P) || !aligned16(dO))
    return set_error(kErrMisaligned, "every buffer must be 16-byte aligned");
  return kOk;
}

// Encodes the tensor maps and enqueues the two kernels on `stream`, with D
// at `dsum` (written by the dQ kernel, or read by both kernels when
// `given_d` is set) and the wait status at `st`. Arguments are already
// checked. With a partial-sum workspace (`part_ws`), tail items may be split
// (plan_units); each kernel with split items is then followed by its combine
// kernel.
// Optional timing events: [0] before the dQ kernel, [1] between the two
// kernels (after the dQ combine), [2] and [3] after the dK/dV kernel (and
// its combine).
template <typename T>
int enqueue_backward(T* dQ, T* dK, T* dV, const T* Q, const T* K, const T* V, const T* P,
                     const T* dO, int M, int N, int D, int H, float* dsum, KernelStatus* st,
                     cudaStream_t stream, cudaEvent_t const* events, bool given_d = false,
                     float* part_ws = nullptr) {
  constexpr bool kBF16 = Elem<T>::kBF16;
  CUtensorMap mQ, mK, mV, mdO, mP;
  if (!encode_fn()) return set_error(kErrNoDriver, "cuTensorMapEncodeTiled is unavailable");
  if (!encode_map(&mQ, kBF16, Q, D, M, H) || !encode_map(&mK, kBF16, K, D, N, H) ||
      !encode_map(&mV, kBF16, V, D, N, H) ||
      !encode_map(&mdO, kBF16, dO, D, M, H) || !encode_map(&mP, kBF16, P, N, M, H))
    return set_error(kErrInvalidArgument, "tensor map encoding failed (M=%d N=%d K_dim=%d heads=%d)",
                     M, N, D, H);
  const uint64_t tmo = effective_timeout_ns();
  auto mark = [&](int k) {
    if (events && events[k]) cudaEventRecord(events[k], stream);
  };
  const int mt = (M + kTile - 1) / kTile;
  int device = 0, sms = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (sms <= 0) sms = 148;
  // both kernels are persistent (one CTA per SM) and walk work units: the
  // dQ kernel's (query tile, head) items over the key tiles, the dK/dV
  // kernel's (key tile, head) items over the query tiles; a last wave that
  // would be at most half full is split into parts (plan_units)
  const int nt = (N + kTile - 1) / kTile;
  const bool can_split = part_ws != nullptr;
  const UnitMap umq = plan_units(mt * H, sms, nt, can_split);
  const dim3 grid_rows(static_cast<unsigned>(umq.units < sms ? umq.units : sms));
  // the dK/dV kernel walks work units: (key tile, head) items, the last
  // wave's split into parts when it would be at most half full
  const UnitMap um = plan_units(nt * H, sms, mt, can_split);
  const dim3 grid_cols(static_cast<unsigned>(um.units < sms ? um.units : sms));
  // combine grids: one thread per (tail item, row, 8 columns); dK/dV rows
  // count twice (dV and dK)
  auto combine_blocks = [&](const UnitMap& u, int rows_per_item) {
    const int64_t tail = (u.units - u.full) / u.parts;
    const int64_t threads = tail * rows_per_item * kTile * (D / 8);
    return dim3(static_cast<unsigned>((threads + kCombineThreads - 1) / kCombineThreads));
  };
  mark(0);
  if (D == 128) {
    if (given_d)
      dq_kernel<T, 128, true><<<grid_rows, DqCfg<128>::kThreads, DqCfg<128>::kSmemBytes, stream>>>(
          mP, mV, mK, mdO, dQ, dsum, M, N, H, umq, part_ws, st, tmo);
    else
      dq_kernel<T, 128><<<grid_rows, DqCfg<128>::kThreads, DqCfg<128>::kSmemBytes, stream>>>(
          mP, mV, mK, mdO, dQ, dsum, M, N, H, umq, part_ws, st, tmo);
    if (umq.parts > 1) {
      if (given_d)
        dq_combine_kernel<T, 128, true><<<combine_blocks(umq, 1), kCombineThreads, 0, stream>>>(
            part_ws, umq, M, dQ, dsum);
      else
        dq_combine_kernel<T, 128, false><<<combine_blocks(umq, 1), kCombineThreads, 0, stream>>>(
            part_ws, umq, M, dQ, dsum);
    }
    mark(1);
    dkv_kernel<T, 128><<<grid_cols, DkvCfg<128>::kThreads, DkvCfg<128>::kSmemBytes, stream>>>(
        mQ, mV, mdO, mP, dsum, dK, dV, M, N, H, um, part_ws, st, tmo);
    if (um.parts > 1)
      dkv_combine_kernel<T, 128><<<combine_blocks(um, 2), kCombineThreads, 0, stream>>>(part_ws, um, N,
                                                                                          dK, dV);
  } else {
    if (given_d)
      dq_kernel<T, 64, true><<<grid_rows, DqCfg<64>::kThreads, DqCfg<64>::kSmemBytes, stream>>>(
          mP, mV, mK, mdO, dQ, dsum, M, N, H, umq, part_ws, st, tmo);
    else
      dq_kernel<T, 64><<<grid_rows, DqCfg<64>::kThreads, DqCfg<64>::kSmemBytes, stream>>>(
          mP, mV, mK, mdO, dQ, dsum, M, N, H, umq, part_ws, st, tmo);
    if (umq.parts > 1) {
      if (given_d)
        dq_combine_kernel<T, 64, true><<<combine_blocks(umq, 1), kCombineThreads, 0, stream>>>(
            part_ws, umq, M, dQ, dsum);
      else
        dq_combine_kernel<T, 64, false><<<combine_blocks(umq, 1), kCombineThreads, 0, stream>>>(
            part_ws, umq, M, dQ, dsum);
    }
    mark(1);
    dkv_kernel<T, 64><<<grid_cols, DkvCfg<64>::kThreads, DkvCfg<64>::kSmemBytes, stream>>>(
        mQ, mV, mdO, mP, dsum, dK, dV, M, N, H, um, part_ws, st, tmo);
    if (um.parts > 1)
      dkv_combine_kernel<T, 64><<<combine_blocks(um, 2), kCombineThreads, 0, stream>>>(part_ws, um, N,
                                                                                         dK, dV);
  }
  mark(2);
  mark(3);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(kErrLaunch, "launch failed: %s", cudaGetErrorString(e));
  return kOk;
}

// Self-test of the bounded-wait machinery: one warp waits on an mbarrier that
// nothing ever arrives on. The wait gives up after `timeout_ns`, records
// (kStatusWaitTimeout, kSelfTestSite) in the status slot and the kernel
// returns normally.
constexpr int kSelfTestSite = 99;
__global__ void wait_selftest_kernel(KernelStatus* status, uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    WaitCtx ctx{reinterpret_cast<volatile int*>(&abort_flag), timeout_ns};
    mbar_wait(&bar, 0, ctx, kSelfTestSite);
    publish_failure(abort_flag, status);
  }
}

// Launches the two kernels on `stream`. When `sync` is set, waits for the
// stream and reports in-kernel wait timeouts as kErrDeviceTimeout.
// `given_d`, when not null, is D = rowsum(P * dP) (fp32, [H][M]) supplied by
// the caller; the dQ kernel then skips the rowsum and the B accumulation.
template <typename T>
int run_backward(T* dQ, T* dK, T* dV, const T* Q, const T* K, const T* V, const T* P,
                 const T* dO, int M, int N, int D, int H, cudaStream_t stream, bool sync,
                 cudaEvent_t const* events = nullptr, const float* given_d = nullptr,
                 bool need_given_d = false) {
  int rc = check_args(dQ, dK, dV, Q, K, V, P, dO, M, N, D, H);
  if (rc != kOk) return rc;
  if (need_given_d && !given_d) return set_error(kErrInvalidArgument, "null D argument");
  if (given_d && (reinterpret_cast<uintptr_t>(given_d) & 3u) != 0)
    return set_error(kErrMisaligned, "D must be float-aligned");
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kErrLaunch, "no current CUDA device");
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0)
    return set_error(kErrUnsupportedDevice, "device %d is sm_%d%d; this library needs sm_100", device,
                     major, minor);
  const size_t rows = static_cast<size_t>(H) * static_cast<size_t>(M);
  // partial-sum workspace for split tail items (at most one wave of parts),
  // shared by the two kernels, which run one after the other: dK/dV slots
  // hold [2][128][K_dim] fp32, dQ slots [2][128][K_dim] + [2][128]
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (sms <= 0) sms = 148;
  const int mtl = (M + kTile - 1) / kTile, ntl = (N + kTile - 1) / kTile;
  const UnitMap umk = plan_units(ntl * H, sms, mtl, true);
  const UnitMap umq = plan_units(mtl * H, sms, ntl, true);
  const size_t slotk = 2 * static_cast<size_t>(kTile) * D, slotq = slotk + 2 * kTile;
  const size_t part_floats = std::max(static_cast<size_t>(umk.units - umk.full) * slotk,
                                      static_cast<size_t>(umq.units - umq.full) * slotq);
  DeviceWorkspace* w = get_workspace<T>(device, given_d ? 0 : rows, part_floats);
  if (!w) return kErrOutOfMemory;

  if (sync) memset(w->host_status, 0, sizeof(KernelStatus));
  rc = enqueue_backward<T>(dQ, dK, dV, Q, K, V, P, dO, M, N, D, H,
                           given_d ? const_cast<float*>(given_d) : w->dsum, w->host_status_dev,
                           stream, events, given_d != nullptr, part_floats > 0 ? w->part : nullptr);
  if (rc != kOk) return rc;
  cudaError_t e = cudaSuccess;
  if (sync) {
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return set_error(kErrLaunch, "kernel failed: %s", cudaGetErrorString(e));
    const KernelStatus stv = read_status(w->host_status);
    if (stv.code != 0) {
      return set_error(kErrDeviceTimeout, "in-kernel wait gave up (code %d, site %d, block %d)",
                       stv.code, stv.where, stv.block);
    }
  }
  return set_error(kOk, "");
}

}  // namespace fmha_sm100
