// Library-wide entry points: device query, status text, version, kernel facts.
#include <cstdio>

#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {

int current_device_facts(DeviceFacts* out) {
  // Facts are cached per device ordinal (attribute queries are cheap, but a
  // launch path should not repeat them on every call); the first query of a
  // device runs under a lock, later ones read the published copy.
  constexpr int kMax = 64;
  static DeviceFacts cache[kMax];
  static std::atomic<bool> ready[kMax];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TCB_ERR_DEVICE;
  if (dev < 0 || dev >= kMax) return TCB_ERR_DEVICE;
  if (!ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[dev].load(std::memory_order_relaxed)) {
      DeviceFacts g;
      g.device = dev;
      if (cudaDeviceGetAttribute(&g.sm_count, cudaDevAttrMultiProcessorCount, dev) !=
              cudaSuccess ||
          cudaDeviceGetAttribute(&g.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                                 dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&g.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&g.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
        return TCB_ERR_DEVICE;
      cache[dev] = g;
      ready[dev].store(true, std::memory_order_release);
    }
  }
  *out = cache[dev];
  return TCB_OK;
}

}  // namespace tcb

using namespace tcb;

extern "C" const char* tcb_strerror(int status) {
  switch (status) {
    case TCB_OK:
      return "ok";
    case TCB_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case TCB_ERR_UNSUPPORTED:
      // Names the matrix format so that a caller classifying messages, as the
      // reference's _unsupported_reason does (bench_tensor.py:94-142), sees a
      // capability rejection rather than a runtime failure.
      return "unsupported matrix format or tile on this device";
    case TCB_ERR_RESOURCE:
      return "configuration exceeds shared memory, tensor memory or register limits";
    case TCB_ERR_LAUNCH:
      return "kernel launch failed";
    case TCB_ERR_DEVICE:
      return "device query failed";
    case TCB_ERR_TIMEOUT:
      return "device-side bounded wait timed out";
    case TCB_ERR_ALIGNMENT:
      return "pointer or size is not aligned as the kernel requires";
    case TCB_ERR_SCRATCH_LIMIT:
      return "problem exceeds the library's fixed scratch array (8 MiB of packed MX scales)";
    default:
      return "unknown status";
  }
}

extern "C" const char* tcb_version(void) { return "tcb 0.1.0 sm_100a"; }

extern "C" int tcb_device_query(int device, tcb_device_props* out) {
  if (out == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return TCB_ERR_DEVICE;
  copy_str(out->name, sizeof(out->name), p.name);
  out->major = p.major;
  out->minor = p.minor;
  out->sm_count = p.multiProcessorCount;
  out->max_smem_per_block = static_cast<int>(p.sharedMemPerBlockOptin);
  out->max_smem_per_sm = static_cast<int>(p.sharedMemPerMultiprocessor);
  out->regs_per_sm = p.regsPerMultiprocessor;
  int clock = 0, mem_clock = 0, bus = 0;
  cudaDeviceGetAttribute(&clock, cudaDevAttrClockRate, device);
  cudaDeviceGetAttribute(&mem_clock, cudaDevAttrMemoryClockRate, device);
  cudaDeviceGetAttribute(&bus, cudaDevAttrGlobalMemoryBusWidth, device);
  out->clock_khz = clock;
  out->mem_clock_khz = mem_clock;
  out->mem_bus_width = bus;
  out->l2_cache_bytes = p.l2CacheSize;
  out->total_mem_bytes = static_cast<long long>(p.totalGlobalMem);
  int previous = 0;
  size_t free_b = 0, total_b = 0;
  if (cudaGetDevice(&previous) == cudaSuccess && cudaSetDevice(device) == cudaSuccess &&
      cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
    out->free_mem_bytes = static_cast<long long>(free_b);
  } else {
    out->free_mem_bytes = -1;
  }
  cudaSetDevice(previous);
  cudaDriverGetVersion(&out->driver_version);
  cudaRuntimeGetVersion(&out->runtime_version);
  return TCB_OK;
}

extern "C" int tcb_kernel_info(int family, int a0, int a1, int a2, int a3, int a4, int a5, int a6,
                               tcb_kernel_info_t* out) {
  if (out == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  *out = tcb_kernel_info_t{};
  switch (family) {
    case TCB_FAMILY_COPY:
      return copy_kernel_info(a0, a1, out);
    case TCB_FAMILY_READ:
      return read_kernel_info(a0, a1, out);
    case TCB_FAMILY_VECTOR:
      return vector_kernel_info(a0, a1, a2, a3, a4, out);
    case TCB_FAMILY_TENSOR:
      return tensor_kernel_info(a0, a1, a2, a3, a4, a5, a6, out);
    case TCB_FAMILY_GEMM_FP4:
      return gemm_kernel_info(a0, a1, a2, out);
    default:
      return TCB_ERR_INVALID_ARGUMENT;
  }
}
