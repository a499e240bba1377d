// extern "C" entry points shared by both libraries (error reporting and the
// wait-timeout setting). Included by exactly one translation unit per
// library, after fmha_bwd_launch.cuh.
#pragma once

#include "fmha_bwd_launch.cuh"

// Exported entry points stay visible when the library is built with
// -fvisibility=hidden (everything else is internal).
#define FMHA_API __attribute__((visibility("default")))

extern "C" {

FMHA_API int fmha_bwd_last_error(void) { return fmha_sm100::error_state().code.load(); }

FMHA_API const char* fmha_bwd_last_error_message(void) { return fmha_sm100::error_state().message; }

FMHA_API int fmha_bwd_work_units(int items, int grid, int len, int allow, int* out) {
  using namespace fmha_sm100;
  if (!out || items < 0 || grid < 0 || len < 0)
    return set_error(kErrInvalidArgument, "work_units: null out or negative size");
  const UnitMap um = plan_units(items, grid, len, allow != 0);
  out[0] = um.full;
  out[1] = um.parts;
  out[2] = um.units;
  return kOk;
}

FMHA_API int fmha_bwd_poll_device_status(void) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return fmha_sm100::kErrLaunch;
  }
  std::lock_guard<std::mutex> g(fmha_sm100::ws_mutex());
  auto& m = fmha_sm100::ws_map();
  auto it = m.find(device);
  if (it == m.end() || it->second.host_status == nullptr) return fmha_sm100::kOk;
  const fmha_sm100::KernelStatus st = fmha_sm100::read_status(it->second.host_status);
  if (st.code == 0) return fmha_sm100::kOk;
  memset(it->second.host_status, 0, sizeof(fmha_sm100::KernelStatus));
  return fmha_sm100::kErrDeviceTimeout;
}

FMHA_API int fmha_bwd_selftest_wait_timeout(int timeout_ms) {
  using namespace fmha_sm100;
  if (timeout_ms <= 0 || timeout_ms > 10000)
    return set_error(kErrInvalidArgument, "timeout_ms=%d outside (0, 10000]", timeout_ms);
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kErrLaunch, "no current CUDA device");
  }
  DeviceWorkspace* w = nullptr;
  {
    std::lock_guard<std::mutex> g(ws_mutex());
    w = &ws_map()[device];
    if (!ensure_status_slot(device, *w)) return kErrOutOfMemory;
  }
  memset(w->host_status, 0, sizeof(KernelStatus));
  wait_selftest_kernel<<<1, 32>>>(w->host_status_dev, static_cast<uint64_t>(timeout_ms) * 1000000ull);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(kErrLaunch, "self-test kernel failed: %s", cudaGetErrorString(e));
  const KernelStatus st = read_status(w->host_status);
  memset(w->host_status, 0, sizeof(KernelStatus));
  if (st.code != kStatusWaitTimeout || st.where != kSelfTestSite)
    return set_error(kErrLaunch, "self-test: expected a recorded wait timeout, got code %d site %d",
                     st.code, st.where);
  return set_error(kOk, "");
}

FMHA_API void fmha_bwd_set_wait_timeout_ms(int ms) {
  fmha_sm100::timeout_override_ns().store(ms > 0 ? static_cast<uint64_t>(ms) * 1000000ull : 0ull);
}

}  // extern "C"
