// Host-side helpers shared by the library's translation units: the per-thread error
// detail of the last failing call, status helpers, and the per-device state (SM count,
// kernel attributes set once per device).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/nvfp4_group_gemm.h"

namespace nvfp4 {

// Detail text of the last failure on this thread (nvfp4_last_error_detail).
extern thread_local std::string g_last_error;

// Record a formatted detail and return `code`.
int fail(int code, const char* fmt, ...);
// NVFP4_ERR_CUDA with the CUDA error's name and text.
int cuda_fail(cudaError_t e, const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag once;
  int status = NVFP4_OK;
  int num_sms = 0;
  int pair_clusters = 0;        // CTA pairs that can be resident at once (plain pair kernel)
  int pair_clusters_gated = 0;  // same for the gated pair kernel
  std::string detail;
};

// The state of the calling thread's current device, initialised on first use (compute
// capability check, kernel shared-memory attributes, occupancy). NVFP4_OK and *out, or the
// failure status with its detail recorded.
int current_device_state(DeviceState** out);

}  // namespace nvfp4
