// Host-side helpers shared by the launch entry points of libtcb.
#pragma once

#include <cstdint>
#include <cstring>
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

inline int launch_status() {
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? TCB_OK : TCB_ERR_LAUNCH;
}

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
