// Host-side helpers shared by the launch entry points of libtcb.
#pragma once

#include <atomic>
#include <climits>
#include <cstdint>
#include <cstring>
#include <mutex>

#include <cuda_runtime.h>

#include "tcb_status.h"

namespace tcb {

struct DeviceFacts {
  int device = -1;
  int sm_count = 0;
  int max_smem_optin = 0;
  int major = 0, minor = 0;
};

// Facts about the current device, cached per device ordinal.  Queried with
// cudaDeviceGetAttribute only (no context-wide side effects, capture-safe).
int current_device_facts(DeviceFacts* out);

// Drop a non-sticky error left by an earlier runtime call, so that the check
// after a launch reports that launch only.
inline void clear_stale_error() { (void)cudaGetLastError(); }

inline int launch_status() {
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? TCB_OK : TCB_ERR_LAUNCH;
}

// Allow `fn` the device's opt-in shared memory minus its static shared
// memory; returns the dynamic bytes a launch may request, or -1.
inline int raise_dynamic_smem(const void* fn, int max_optin) {
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, fn) != cudaSuccess) {
    clear_stale_error();
    return -1;
  }
  const int cap = max_optin - static_cast<int>(attr.sharedSizeBytes);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, cap) != cudaSuccess) {
    clear_stale_error();
    return -1;
  }
  return cap;
}

// A per-device integer computed once (for example a kernel's dynamic
// shared-memory allowance).  Thread-safe: the first caller for a device runs
// `compute` under a lock, later callers read the published value.
class DeviceIntCache {
 public:
  DeviceIntCache() {
    for (auto& v : value_) v.store(kUnset, std::memory_order_relaxed);
  }
  template <typename F>
  int get(int device, F compute) {
    if (device < 0 || device >= kMaxDevices) return -1;
    int v = value_[device].load(std::memory_order_acquire);
    if (v != kUnset) return v;
    std::lock_guard<std::mutex> lock(mu_);
    v = value_[device].load(std::memory_order_relaxed);
    if (v == kUnset) {
      v = compute();
      value_[device].store(v, std::memory_order_release);
    }
    return v;
  }

 private:
  static constexpr int kMaxDevices = 64;
  static constexpr int kUnset = INT_MIN;
  std::atomic<int> value_[kMaxDevices];
  std::mutex mu_;
};

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline bool is_pow2(long long v) { return v > 0 && (v & (v - 1)) == 0; }

// Copy a C string into a fixed buffer, always terminated.
inline void copy_str(char* dst, size_t cap, const char* src) {
  if (cap == 0) return;
  std::strncpy(dst, src, cap - 1);
  dst[cap - 1] = '\0';
}

}  // namespace tcb
