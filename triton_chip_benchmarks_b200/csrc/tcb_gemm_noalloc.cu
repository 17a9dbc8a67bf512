// MX FP4 GEMM for callers that cannot allocate device memory.
//
// tcb_gemm reads MX FP4 scales in a packed layout that a caller normally
// builds once, in buffers it allocates (tcb_mx_scales_packed_bytes +
// tcb_mx_scales_pack).  Some callers cannot do that: a plugin whose host
// framework owns every device allocation through its own pool and forbids
// direct cudaMalloc, or a caller on a latency-critical path where an
// allocation (and the device synchronisation cudaFree implies) is not
// allowed.  tcb_gemm_mxf4_noalloc takes the scales in the plain [rows][K/32]
// E8M0 layout and packs them into a fixed scratch array that lives in this
// library's device image, so the call allocates nothing.
//
// The scratch array is a file-scope __device__ variable: every device that
// loads this library's code holds kNoAllocScratchBytes for it until the
// process exits.  In host code its name is only a host-side stand-in, never
// a device address; the address comes from cudaGetSymbolAddress, queried
// once per device (with that device current) on the first call made on it.
#include <atomic>
#include <mutex>

#include "tcb_host.h"

namespace tcb {
namespace {

// Packed scales of A and of B together (each rounded up to 256 bytes) must
// fit here.  8 MiB holds, for example, M = N = 8192 at K = 8192 (2 MiB per
// operand) and M = N = 16384 at K = 8192 (4 MiB per operand).
constexpr long long kNoAllocScratchBytes = 8ll << 20;

static __device__ __align__(256) uint8_t g_mxf4_scale_scratch[kNoAllocScratchBytes];

// Device address of the scratch array on the current device.  The first call
// on a device resolves it under a lock; later calls read the cached value.
int scratch_address(uint8_t** out) {
  constexpr int kMaxDevices = 64;
  static std::atomic<uint8_t*> cached[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    clear_stale_error();
    return TCB_ERR_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return TCB_ERR_DEVICE;
  uint8_t* p = cached[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(mu);
    p = cached[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void* addr = nullptr;
      const cudaError_t err = cudaGetSymbolAddress(&addr, g_mxf4_scale_scratch);
      if (err != cudaSuccess || addr == nullptr) {
        clear_stale_error();
        return TCB_ERR_DEVICE;
      }
      p = static_cast<uint8_t*>(addr);
      cached[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return TCB_OK;
}

}  // namespace
}  // namespace tcb

using namespace tcb;

extern "C" int tcb_gemm_mxf4_noalloc(const void* A, const void* B, const void* SA,
                                     const void* SB, void* C, int M, int N, int K, int blocks,
                                     int* status_dev, tcb_stream_t stream) {
  if (A == nullptr || B == nullptr || SA == nullptr || SB == nullptr || C == nullptr || M <= 0 ||
      N <= 0 || K <= 0 || blocks < 0)
    return TCB_ERR_INVALID_ARGUMENT;
  // One E8M0 scale per 32 K elements; a row of E2M1 codes must also be a
  // whole number of 16-byte units, which K % 32 == 0 gives.
  if (K % 32 != 0) return TCB_ERR_UNSUPPORTED;
  const int groups = K / 32;
  const long long a_bytes = tcb_mx_scales_packed_bytes(M, groups);
  const long long b_offset = (a_bytes + 255) / 256 * 256;
  const long long b_bytes = tcb_mx_scales_packed_bytes(N, groups);
  if (b_offset + b_bytes > kNoAllocScratchBytes) return TCB_ERR_SCRATCH_LIMIT;
  uint8_t* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != TCB_OK) return rc;
  // Each pack rewrites every byte of its region (padding included), so the
  // previous call's contents never leak into this one.  The packs and the
  // GEMM run in order on `stream`.
  if ((rc = tcb_mx_scales_pack(SA, scratch, M, groups, stream)) != TCB_OK) return rc;
  if ((rc = tcb_mx_scales_pack(SB, scratch + b_offset, N, groups, stream)) != TCB_OK) return rc;
  return tcb_gemm(TCB_T_MXF4, A, B, scratch, scratch + b_offset, C, M, N, K, blocks, status_dev,
                  stream);
}
