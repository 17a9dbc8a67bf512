// Device copy and read bandwidth probes (sm_100a).
//
// copy: dst = src over a byte range.  Two kernels:
//   * LDG128 - register copy, one CTA per piece of THREADS x 32 bytes: each
//     thread loads its 32 bytes (one 256-bit vector when both pointers are
//     32-byte aligned, else two 16-byte vectors a CTA width apart, both in
//     flight) and stores them.  The CTA size is a template parameter for the
//     common sizes.  An explicit grid size walks the pieces grid-stride
//     instead (a second kernel).
//     Measured on B200 (2-4 GiB): 768-thread CTAs, two resident per SM (48 KB
//     of loads in flight per SM), copy at 7.0-7.1 TB/s; 1024 threads 7.0,
//     128-512 threads 6.92-6.96, one or three 16-byte vectors per thread
//     6.16-6.97; the same code inside a grid-stride loop (even one that runs
//     once) 6.57 at 768 threads, persistent grids of 2-16 CTAs per SM
//     5.9-6.4.  256-bit vectors hold 7.08-7.11 at every source/destination
//     offset tried, where two 16-byte vectors dip to 6.96.  Any shared memory
//     on the CTA costs L1 capacity, which holds the in-flight loads: the same
//     pieces with 48 KB of shared memory per CTA copy at 6.2 TB/s, which is
//     also where the bulk-copy ring below (6.6-6.7 TB/s) loses.
//   * BULK   - the bulk-copy engine: one lane per CTA moves CHUNK-byte pieces
//     global -> shared -> global through a ring of STAGES buffers; completion
//     of loads is tracked by mbarriers, of stores by bulk groups.
// read: per-block FP32 sum of a block of elements into a sink word, the
//   streaming-read companion pattern (16-byte .cg loads).
//
// Counterparts in the reference suite: copy_kernel / launch_copy
// (bench_bandwidth.py:36-47) and read_kernel / launch_read
// (bench_bandwidth.py:50-67).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "tcb_device.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

constexpr int kCopyVectors = 2;       // 16-byte vectors per thread of the LDG128 kernel
constexpr int kCopyDefaultThreads = 768;
constexpr int kBulkChunk = 32768;
constexpr int kBulkMaxStages = 8;
constexpr int kBulkDefaultStages = 2;

__device__ __forceinline__ uint4 ld_stream_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_stream_v4(uint4* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Copy of the trailing bytes that do not fill a 16-byte vector.
__device__ __forceinline__ void copy_tail(const unsigned char* src, unsigned char* dst,
                                          size_t first, size_t bytes) {
  if (blockIdx.x == 0) {
    for (size_t i = first + threadIdx.x; i < bytes; i += blockDim.x) dst[i] = src[i];
  }
}

struct alignas(32) Vec32 {
  uint32_t w[8];
};

__device__ __forceinline__ Vec32 ld_v8(const Vec32* p) {
  Vec32 v;
  asm volatile("ld.global.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]),
                 "=r"(v.w[5]), "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v8(Vec32* p, const Vec32& v) {
  asm volatile("st.global.v8.u32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v.w[0]),
               "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]),
               "r"(v.w[7])
               : "memory");
}

// One piece of THREADS x 32 bytes per CTA over nvec 16-byte vectors.
// THREADS = 0: the CTA size is blockDim.x.  WIDE: 256-bit vectors (both
// pointers 32-byte aligned); an odd last 16-byte vector goes to the thread
// just past the 256-bit ones.
template <int THREADS, bool WIDE>
__global__ void __launch_bounds__(THREADS ? THREADS : 1024)
    copy_piece_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t nvec) {
  const size_t threads = THREADS ? THREADS : blockDim.x;
  if constexpr (WIDE) {
    const size_t i = static_cast<size_t>(blockIdx.x) * threads + threadIdx.x;
    const size_t n32 = nvec >> 1;
    if (i < n32)
      st_v8(reinterpret_cast<Vec32*>(dst) + i, ld_v8(reinterpret_cast<const Vec32*>(src) + i));
    else if (i == n32 && (nvec & 1))
      st_stream_v4(dst + nvec - 1, ld_stream_v4(src + nvec - 1));
  } else {
    const size_t i = static_cast<size_t>(blockIdx.x) * threads * kCopyVectors + threadIdx.x;
    uint4 v[kCopyVectors];
#pragma unroll
    for (int u = 0; u < kCopyVectors; ++u)
      if (i + u * threads < nvec) v[u] = ld_stream_v4(src + i + u * threads);
#pragma unroll
    for (int u = 0; u < kCopyVectors; ++u)
      if (i + u * threads < nvec) st_stream_v4(dst + i + u * threads, v[u]);
  }
}

// The same pieces walked grid-stride by a grid of any size.
__global__ void __launch_bounds__(1024)
    copy_stride_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t nvec) {
  const size_t piece = static_cast<size_t>(blockDim.x) * kCopyVectors;
  for (size_t p = blockIdx.x; p * piece < nvec; p += gridDim.x) {
    const size_t i = p * piece + threadIdx.x;
    uint4 v[kCopyVectors];
#pragma unroll
    for (int u = 0; u < kCopyVectors; ++u)
      if (i + u * blockDim.x < nvec) v[u] = ld_stream_v4(src + i + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < kCopyVectors; ++u)
      if (i + u * blockDim.x < nvec) st_stream_v4(dst + i + u * blockDim.x, v[u]);
  }
}

using PieceFn = void (*)(const uint4*, uint4*, size_t);

// The one-shot kernel for a CTA size (compile-time for the common sizes).
PieceFn copy_piece_fn(int threads, bool wide) {
  switch (threads) {
    case 256: return wide ? copy_piece_kernel<256, true> : copy_piece_kernel<256, false>;
    case 512: return wide ? copy_piece_kernel<512, true> : copy_piece_kernel<512, false>;
    case 768: return wide ? copy_piece_kernel<768, true> : copy_piece_kernel<768, false>;
    case 1024: return wide ? copy_piece_kernel<1024, true> : copy_piece_kernel<1024, false>;
    default: return wide ? copy_piece_kernel<0, true> : copy_piece_kernel<0, false>;
  }
}

__global__ void copy_bytes_kernel(const unsigned char* __restrict__ src,
                                  unsigned char* __restrict__ dst, size_t bytes) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < bytes;
       i += stride)
    dst[i] = src[i];
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t size,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(smem_dst)),
      "l"(src), "r"(size), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, const void* smem_src, uint32_t size) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(smem_src)), "r"(size)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Chunk k of this CTA covers bytes [off, off+size) of the 16-byte aligned body.
__device__ __forceinline__ void bulk_chunk(size_t body, long long k, size_t* off, uint32_t* size) {
  const size_t start = (static_cast<size_t>(blockIdx.x) + static_cast<size_t>(k) * gridDim.x) *
                       static_cast<size_t>(kBulkChunk);
  const size_t left = body - start;
  *off = start;
  *size = static_cast<uint32_t>(left < kBulkChunk ? left : kBulkChunk);
}

__global__ void __launch_bounds__(32)
    copy_bulk_kernel(const unsigned char* __restrict__ src, unsigned char* __restrict__ dst,
                     size_t bytes, int stages, int* status) {
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ __align__(8) uint64_t bars[kBulkMaxStages];
  const size_t body = bytes & ~static_cast<size_t>(15);
  const size_t nchunks_total = (body + kBulkChunk - 1) / kBulkChunk;
  const long long mine =
      blockIdx.x < nchunks_total
          ? static_cast<long long>((nchunks_total - 1 - blockIdx.x) / gridDim.x + 1)
          : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    const long long prologue = mine < stages ? mine : stages;
    for (long long k = 0; k < prologue; ++k) {
      size_t off;
      uint32_t size;
      bulk_chunk(body, k, &off, &size);
      mbar_arrive_expect_tx(&bars[k], size);
      bulk_load(ring + k * kBulkChunk, src + off, size, &bars[k]);
    }
    for (long long k = 0; k < mine; ++k) {
      const int s = static_cast<int>(k % stages);
      const uint32_t phase = static_cast<uint32_t>((k / stages) & 1);
      if (!mbar_wait(&bars[s], phase)) {
        report_status(status, TCB_ERR_TIMEOUT);
        break;
      }
      size_t off;
      uint32_t size;
      bulk_chunk(body, k, &off, &size);
      bulk_store(dst + off, ring + s * kBulkChunk, size);
      bulk_commit();
      // Refill the stage whose store was issued one step earlier, once that
      // store has finished reading its shared-memory buffer.
      const long long refill = k - 1 + stages;
      if (k >= 1 && refill < mine) {
        bulk_wait_read<1>();
        const int rs = static_cast<int>((k - 1) % stages);
        size_t roff;
        uint32_t rsize;
        bulk_chunk(body, refill, &roff, &rsize);
        mbar_arrive_expect_tx(&bars[rs], rsize);
        bulk_load(ring + rs * kBulkChunk, src + roff, rsize, &bars[rs]);
      }
    }
    bulk_wait_all();
  }
  copy_tail(src, dst, body, bytes);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ uint4 ld_cg_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// A thread's VPT vectors (tid + u x blockDim.x), all loads issued before the
// first sum, added to the partials in the same order as the loop form.
template <typename T, int VPT>
__device__ __forceinline__ void sum_vectors(const uint4* vsrc, float (&part)[16 / sizeof(T)]) {
  constexpr int kVec = 16 / sizeof(T);
  uint4 raw[VPT];
#pragma unroll
  for (int u = 0; u < VPT; ++u) raw[u] = ld_cg_v4(vsrc + threadIdx.x + u * blockDim.x);
#pragma unroll
  for (int u = 0; u < VPT; ++u) {
    const T* vals = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
    for (int j = 0; j < kVec; ++j) part[j] += to_f32(vals[j]);
  }
}

// One CTA sums `block_elems` consecutive elements.  Each thread accumulates
// its 16-byte vectors lane-wise into independent FP32 partials, then the
// CTA reduces them with warp shuffles and one shared-memory pass.  When a
// whole block splits into 1, 2, 4 or 8 vectors per thread (`vec_per_thread`,
// computed once on the host; 0 otherwise) all of a thread's loads are issued
// at once, with no per-CTA set-up arithmetic before them; other blocks, and
// the partial last block, loop.  Measured on B200 (2 GiB fp32, random data,
// bare harness): 7.49 TB/s at 4096 elements on 256 threads, 7.51 at 16384 on
// 1024; a 64-bit division per CTA ahead of the loads cost about 0.4 %.
template <typename T>
__global__ void __launch_bounds__(1024)
    read_sum_kernel(const T* __restrict__ src, long long elements, float* __restrict__ sink,
                    int block_elems, int vec_per_thread) {
  constexpr int kVec = 16 / sizeof(T);
  __shared__ float warp_sums[32];
  const long long base = static_cast<long long>(blockIdx.x) * block_elems;
  const uint4* vsrc = reinterpret_cast<const uint4*>(src + base);
  float part[kVec];
#pragma unroll
  for (int j = 0; j < kVec; ++j) part[j] = 0.f;
  if (vec_per_thread != 0 && elements - base >= block_elems) {
    switch (vec_per_thread) {
      case 1: sum_vectors<T, 1>(vsrc, part); break;
      case 2: sum_vectors<T, 2>(vsrc, part); break;
      case 4: sum_vectors<T, 4>(vsrc, part); break;
      default: sum_vectors<T, 8>(vsrc, part); break;
    }
  } else {
    long long count = elements - base;
    if (count > block_elems) count = block_elems;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
    const long long nvec = vec_ok ? count / kVec : 0;
    for (long long v = threadIdx.x; v < nvec; v += blockDim.x) {
      uint4 raw = ld_cg_v4(vsrc + v);
      const T* vals = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < kVec; ++j) part[j] += to_f32(vals[j]);
    }
    for (long long e = nvec * kVec + threadIdx.x; e < count; e += blockDim.x)
      part[0] += to_f32(src[base + e]);
  }
  float total = 0.f;
#pragma unroll
  for (int j = 0; j < kVec; ++j) total += part[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_sums[warp] = total;
  __syncthreads();
  if (warp == 0) {
    const int nwarps = blockDim.x >> 5;
    float t = lane < nwarps ? warp_sums[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) sink[blockIdx.x] = t;
  }
}

}  // namespace

int copy_bulk_stages(int requested) {
  return requested == 0 ? kBulkDefaultStages : requested;
}
int copy_bulk_smem_bytes(int stages) { return stages * kBulkChunk; }

}  // namespace tcb

using namespace tcb;

extern "C" int tcb_copy(const void* src, void* dst, size_t bytes, int variant, int blocks,
                        int threads, int* status_dev, tcb_stream_t stream) {
  if (bytes == 0) return TCB_OK;
  if (src == nullptr || dst == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  if (variant != TCB_COPY_LDG128 && variant != TCB_COPY_BULK) return TCB_ERR_INVALID_ARGUMENT;
  if (blocks < 0 || threads < 0) return TCB_ERR_INVALID_ARGUMENT;
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  clear_stale_error();
  const bool vec_ok = aligned(src, 16) && aligned(dst, 16);
  if (!vec_ok) {
    copy_bytes_kernel<<<facts.sm_count * 8, 256, 0, s>>>(
        static_cast<const unsigned char*>(src), static_cast<unsigned char*>(dst), bytes);
    return launch_status();
  }
  if (variant == TCB_COPY_LDG128) {
    if (threads == 0) threads = kCopyDefaultThreads;
    if (threads < 32 || threads > 1024 || threads % 32) return TCB_ERR_INVALID_ARGUMENT;
    const size_t nvec = bytes >> 4;
    const size_t piece_vecs = static_cast<size_t>(threads) * kCopyVectors;
    const size_t pieces = (nvec + piece_vecs - 1) / piece_vecs;
    if (pieces > 0x7fffffffULL) return TCB_ERR_INVALID_ARGUMENT;
    if (pieces > 0) {
      const auto* s4 = static_cast<const uint4*>(src);
      auto* d4 = static_cast<uint4*>(dst);
      if (blocks > 0 && static_cast<size_t>(blocks) < pieces) {
        copy_stride_kernel<<<blocks, threads, 0, s>>>(s4, d4, nvec);
      } else {
        const bool wide = aligned(src, 32) && aligned(dst, 32);
        copy_piece_fn(threads, wide)<<<static_cast<unsigned>(pieces), threads, 0, s>>>(s4, d4,
                                                                                       nvec);
      }
    }
    if (bytes & 15) {
      const size_t body = nvec << 4;
      copy_bytes_kernel<<<1, 32, 0, s>>>(static_cast<const unsigned char*>(src) + body,
                                         static_cast<unsigned char*>(dst) + body, bytes & 15);
    }
    return launch_status();
  }
  // Bulk-copy engine: one warp per CTA (lane 0 drives the ring); `threads`
  // selects the ring depth in 32 KiB chunks.
  const int stages = copy_bulk_stages(threads);
  if (stages < 2 || stages > kBulkMaxStages) return TCB_ERR_INVALID_ARGUMENT;
  const int smem = copy_bulk_smem_bytes(stages);
  static DeviceIntCache cap_cache;
  const int cap = cap_cache.get(facts.device, [&] {
    return raise_dynamic_smem(reinterpret_cast<const void*>(copy_bulk_kernel), facts.max_smem_optin);
  });
  if (cap < smem) return TCB_ERR_RESOURCE;
  if (blocks == 0) blocks = facts.sm_count * 2;
  copy_bulk_kernel<<<blocks, 32, smem, s>>>(static_cast<const unsigned char*>(src),
                                            static_cast<unsigned char*>(dst), bytes, stages,
                                            status_dev);
  return launch_status();
}

extern "C" int tcb_read(const void* src, int dtype, long long elements, float* sink,
                        int block_elems, int threads, tcb_stream_t stream) {
  if (elements == 0) return TCB_OK;
  if (src == nullptr || sink == nullptr || elements < 0) return TCB_ERR_INVALID_ARGUMENT;
  if (!is_pow2(block_elems) || block_elems < 256 || block_elems > 65536)
    return TCB_ERR_INVALID_ARGUMENT;
  if (threads == 0) threads = 256;
  if (threads < 32 || threads > 1024 || threads % 32) return TCB_ERR_INVALID_ARGUMENT;
  const long long grid = (elements + block_elems - 1) / block_elems;
  if (grid > 0x7fffffffLL) return TCB_ERR_INVALID_ARGUMENT;
  if (dtype != TCB_READ_FP32 && dtype != TCB_READ_FP16 && dtype != TCB_READ_BF16)
    return TCB_ERR_INVALID_ARGUMENT;
  // 16-byte vectors per thread of a whole block, when the block splits evenly
  // into 1, 2, 4 or 8 of them and the source is 16-byte aligned; else 0 (loop).
  const int vec_elems = dtype == TCB_READ_FP32 ? 4 : 8;
  int vpt = block_elems % (vec_elems * threads) == 0 ? block_elems / (vec_elems * threads) : 0;
  if ((vpt != 1 && vpt != 2 && vpt != 4 && vpt != 8) || !aligned(src, 16)) vpt = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  clear_stale_error();
  switch (dtype) {
    case TCB_READ_FP32:
      read_sum_kernel<float><<<static_cast<unsigned>(grid), threads, 0, s>>>(
          static_cast<const float*>(src), elements, sink, block_elems, vpt);
      break;
    case TCB_READ_FP16:
      read_sum_kernel<__half><<<static_cast<unsigned>(grid), threads, 0, s>>>(
          static_cast<const __half*>(src), elements, sink, block_elems, vpt);
      break;
    case TCB_READ_BF16:
      read_sum_kernel<__nv_bfloat16><<<static_cast<unsigned>(grid), threads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(src), elements, sink, block_elems, vpt);
      break;
    default:
      return TCB_ERR_INVALID_ARGUMENT;
  }
  return launch_status();
}

// Kernel facts for tcb_kernel_info (registry hooks).
namespace tcb {
int copy_kernel_info(int variant, int threads, tcb_kernel_info_t* out) {
  cudaFuncAttributes attr;
  const void* fn = variant == TCB_COPY_BULK
                       ? reinterpret_cast<const void*>(copy_bulk_kernel)
                       : reinterpret_cast<const void*>(
                             copy_piece_fn(threads ? threads : kCopyDefaultThreads, true));
  if (cudaFuncGetAttributes(&attr, fn) != cudaSuccess) return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes =
      variant == TCB_COPY_BULK ? copy_bulk_smem_bytes(copy_bulk_stages(threads)) : 0;
  out->threads_per_block = variant == TCB_COPY_BULK ? 32 : (threads ? threads : kCopyDefaultThreads);
  out->tensor_core = 0;
  copy_str(out->instruction, sizeof(out->instruction),
           variant == TCB_COPY_BULK
               ? "cp.async.bulk.shared::cluster.global / cp.async.bulk.global.shared::cta"
               : "ld.global.v8.u32 / st.global.v8.u32 (32-byte aligned; else "
                 "ld.global.nc.v4.u32 / st.global.cs.v4.u32)");
  copy_str(out->execution_kind, sizeof(out->execution_kind), "memory");
  return TCB_OK;
}

int read_kernel_info(int dtype, int threads, tcb_kernel_info_t* out) {
  cudaFuncAttributes attr;
  const void* fn = dtype == TCB_READ_FP16   ? reinterpret_cast<const void*>(read_sum_kernel<__half>)
                   : dtype == TCB_READ_BF16 ? reinterpret_cast<const void*>(
                                                  read_sum_kernel<__nv_bfloat16>)
                                            : reinterpret_cast<const void*>(read_sum_kernel<float>);
  if (cudaFuncGetAttributes(&attr, fn) != cudaSuccess) return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = 0;
  out->threads_per_block = threads ? threads : 256;
  out->tensor_core = 0;
  copy_str(out->instruction, sizeof(out->instruction), "ld.global.cg.v4.u32");
  copy_str(out->execution_kind, sizeof(out->execution_kind), "memory");
  return TCB_OK;
}
}  // namespace tcb
