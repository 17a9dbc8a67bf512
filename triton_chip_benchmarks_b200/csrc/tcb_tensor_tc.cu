// Resident-operand tensor-core probe on 5th-generation tensor cores (sm_100a).
//
// One CTA of 128 threads per tile.  The CTA
//   1. allocates its share of tensor memory (512 / blocks_per_sm columns),
//   2. stages A[tile_m x K] and B_c[tile_n x K] (c < chains) into shared
//      memory once with 2-D TMA tile loads, K-major, swizzled per 128-, 64- or
//      32-byte panel (the shared-memory matrix descriptor's canonical layout),
//   3. for MX FP4 writes the E8M0 scale factors into tensor memory,
//   4. lets one thread issue `iterations` x (tile_m/128) x chains x (K/MMA_K)
//      tcgen05.mma instructions (M=128, N=tile_n) that accumulate in tensor
//      memory, committed to an mbarrier,
//   5. reads the accumulators back with tcgen05.ld and stores C.
// A 256-row tile is two M=128 accumulators.  A 64-row tile (not MX FP4) is one
// M=64 accumulator, which tensor memory holds 16 rows per 32-lane
// sub-partition: row 16w + i in lane 32w + i, i < 16.  When the accumulators plus the
// scale factors do not fit the CTA's tensor-memory share at once, the
// (half, chain) accumulator groups run in consecutive passes; every group
// still receives exactly `iterations` accumulations of its tile product.
//
// Counterparts in the reference suite: _tensor_peak_kernel
// (bench_tensor.py:406-449) and _tensor_peak_scaled_kernel
// (bench_tensor.py:452-488), launched by _launch_peak (bench_tensor.py:581-600).
#include <cudaTypedefs.h>

#include "tcb_device.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

enum Kind : int { kF16 = 0, kBF16 = 1, kTF32 = 2, kI8 = 3, kE4M3 = 4, kMXF4 = 5 };

constexpr int kThreads = 128;
constexpr int kMmaKBytes = 32;  // every tcgen05.mma kind here consumes 32 bytes of K per row
constexpr int kSmemPerSM = 233472;

struct TcArgs {
  const uint8_t* sa;  // MX FP4 scales [blocks][tile_m][tile_k/32]
  const uint8_t* sb;  // MX FP4 scales [blocks][tile_n][tile_k/32]
  void* c;            // [chains][blocks][tile_m][tile_n], 32-bit elements
  int* status;
  int blocks, tile_m, tile_n, kbytes, panel, chains, iterations;
  int halves, ksteps, groups, groups_per_pass, tmem_cols, sf_groups;
  int mma_m;        // rows of one accumulator: 128, or 64 for a 64-row tile
  uint32_t layout;  // descriptor swizzle code: 2 = 128B, 4 = 64B, 6 = 32B
  uint32_t idesc;   // instruction descriptor
};

template <int KIND>
__device__ __forceinline__ void mma_issue(uint32_t d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate, uint32_t tsfa,
                                          uint32_t tsfb) {
  if constexpr (KIND == kF16 || KIND == kBF16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == kTF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == kI8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == kE4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], "
        "p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  }
}

// Maximum (half, chain) accumulator groups resident at once: 2 halves x 2 chains.
constexpr int kMaxGroups = 4;

// Single-thread MMA issue over the resident tiles for one pass, specialised on
// the K-steps per tile (KSTEPS) and the panel width (PANEL bytes) so that the
// per-MMA work is an add on the descriptor's address field and the issue.
// Operand j of group gi starts at a_lo[gi] (16-byte units); k-step s of a
// K-major operand with `rows` rows sits at panel s*32/PANEL, column
// (s*32) % PANEL.
template <int KIND, int KSTEPS, int PANEL>
__device__ __forceinline__ void issue_pass(const uint32_t (&d)[kMaxGroups],
                                           const uint32_t (&a_lo)[kMaxGroups],
                                           const uint32_t (&b_lo)[kMaxGroups],
                                           const uint32_t (&sfa)[kMaxGroups], uint32_t sfb,
                                           int groups, int rows_a, int rows_b, int iterations,
                                           uint64_t desc_const, uint32_t idesc,
                                           uint32_t sf_step_cols) {
  uint32_t a_off[KSTEPS], b_off[KSTEPS];
#pragma unroll
  for (int s = 0; s < KSTEPS; ++s) {
    constexpr int kStepsPerPanel = PANEL / kMmaKBytes;
    const int p = s / kStepsPerPanel, w = (s % kStepsPerPanel) * kMmaKBytes;
    a_off[s] = static_cast<uint32_t>(p * rows_a * PANEL + w) >> 4;
    b_off[s] = static_cast<uint32_t>(p * rows_b * PANEL + w) >> 4;
  }
#pragma unroll 1
  for (int it = 0; it < iterations; ++it) {
#pragma unroll
    for (int gi = 0; gi < kMaxGroups; ++gi) {
      if (gi < groups) {
#pragma unroll
        for (int s = 0; s < KSTEPS; ++s) {
          const uint64_t ad = desc_const | (a_lo[gi] + a_off[s]);
          const uint64_t bd = desc_const | (b_lo[gi] + b_off[s]);
          mma_issue<KIND>(d[gi], ad, bd, idesc, s != 0 || it != 0,
                          sfa[gi] + s * sf_step_cols, sfb + s * sf_step_cols);
        }
      }
    }
  }
}

template <int KIND, int KSTEPS, int PANEL>
__global__ void __launch_bounds__(kThreads, 1)
    tc_peak_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b, const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_load;
  __shared__ __align__(8) uint64_t bar_mma;
  __shared__ uint32_t tmem_slot;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x;
  const int M = args.tile_m, N = args.tile_n, panel = PANEL;
  const int panels = args.kbytes / PANEL;
  uint8_t* sA = smem;
  uint8_t* sB = smem + M * args.kbytes;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, static_cast<uint32_t>(args.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_slot;

  // 2. Operands: one TMA tile per 128/64/32-byte K panel of A and of each B_c.
  if (threadIdx.x == 0) {
    const uint32_t bytes = static_cast<uint32_t>((M + args.chains * N) * args.kbytes);
    mbar_arrive_expect_tx(&bar_load, bytes);
    for (int p = 0; p < panels; ++p)
      tma_load_2d(sA + p * M * panel, &map_a, p * panel, blk * M, &bar_load);
    for (int c = 0; c < args.chains; ++c)
      for (int p = 0; p < panels; ++p)
        tma_load_2d(sB + (c * panels + p) * N * panel, &map_b, p * panel,
                    (c * args.blocks + blk) * N, &bar_load);
  }

  // 3. MX scale factors.  For k-step s the A factors of half h sit in 4
  // columns (row 32j+i in lane i of column j, replicated in all four lane
  // quarters) and the B factors in tile_n/32 columns the same way; the two
  // factors of a 64-element step fill bytes 0 and 1 (repeated in 2 and 3).
  const int sf_base = args.groups_per_pass * N;
  const int sf_step_cols = 4 * args.halves + N / 32;
  if constexpr (KIND == kMXF4) {
    const int groups_k = args.ksteps * 2;
    const uint8_t* sa = args.sa + static_cast<size_t>(blk) * M * groups_k;
    const uint8_t* sb = args.sb + static_cast<size_t>(blk) * N * groups_k;
    const uint32_t lane_base = tbase + ((32u * warp) << 16);
    for (int s = 0; s < args.ksteps; ++s) {
      const int col0 = sf_base + s * sf_step_cols;
      for (int h = 0; h < args.halves; ++h)
        for (int j = 0; j < 4; ++j) {
          const uint8_t* r = sa + (h * 128 + 32 * j + lane) * groups_k + 2 * s;
          const uint32_t v = r[0] | (r[1] << 8);
          tmem_st_1col(lane_base + col0 + 4 * h + j, v | (v << 16));
        }
      for (int j = 0; j < N / 32; ++j) {
        const uint8_t* r = sb + (32 * j + lane) * groups_k + 2 * s;
        const uint32_t v = r[0] | (r[1] << 8);
        tmem_st_1col(lane_base + col0 + 4 * args.halves + j, v | (v << 16));
      }
    }
    tmem_wait_st();
  }

  bool ok = mbar_wait(&bar_load, 0);
  if (!ok) report_status(args.status, TCB_ERR_TIMEOUT);
  tc_fence_before();
  ok = __syncthreads_and(ok) != 0;
  tc_fence_after();

  const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB);
  const uint64_t desc_const = smem_desc(0, 16, static_cast<uint32_t>(8 * PANEL), args.layout);
  const int passes = (args.groups + args.groups_per_pass - 1) / args.groups_per_pass;
  for (int pass = 0; ok && pass < passes; ++pass) {
    const int g0 = pass * args.groups_per_pass;
    const int g1 = min(args.groups, g0 + args.groups_per_pass);
    // 4. Single-thread MMA issue over the resident tiles.
    if (warp == 0) {
      if (lane == 0) {
        tc_fence_after();
        uint32_t d[kMaxGroups], a_lo[kMaxGroups], b_lo[kMaxGroups], sfa[kMaxGroups];
#pragma unroll
        for (int gi = 0; gi < kMaxGroups; ++gi) {
          const int g = min(g0 + gi, args.groups - 1);
          const int c = g / args.halves, h = g - c * args.halves;
          d[gi] = tbase + static_cast<uint32_t>(gi * N);
          a_lo[gi] = (a0 + static_cast<uint32_t>(h * 128 * PANEL)) >> 4;
          b_lo[gi] = (b0 + static_cast<uint32_t>(c * panels * N * PANEL)) >> 4;
          sfa[gi] = tbase + static_cast<uint32_t>(sf_base + 4 * h);
        }
        const uint32_t sfb = tbase + static_cast<uint32_t>(sf_base + 4 * args.halves);
        issue_pass<KIND, KSTEPS, PANEL>(d, a_lo, b_lo, sfa, sfb, g1 - g0, M, N, args.iterations,
                                        desc_const, args.idesc,
                                        static_cast<uint32_t>(sf_step_cols));
        tc_commit(&bar_mma);
      }
      __syncwarp();
    }
    bool done = mbar_wait(&bar_mma, static_cast<uint32_t>(pass & 1));
    if (!done) {
      report_status(args.status, TCB_ERR_TIMEOUT);
      // Give in-flight MMAs one more bounded window before tensor memory is freed.
      mbar_wait(&bar_mma, static_cast<uint32_t>(pass & 1));
    }
    tc_fence_after();
    ok = __syncthreads_and(done) != 0;
    if (!ok) break;

    // 5. Epilogue: warp w reads lanes 32w..32w+31 of each accumulator, which
    //    hold rows 32w..32w+31 (M=128) or, in lanes 32w..32w+15, rows
    //    16w..16w+15 (M=64).  Every lane takes part in the warp-wide loads.
    const bool m64 = args.mma_m == 64;
    const bool live = !m64 || lane < 16;
    for (int g = g0; g < g1; ++g) {
      const int c = g / args.halves, h = g - c * args.halves;
      const int row = m64 ? 16 * warp + (lane & 15) : h * 128 + 32 * warp + lane;
      uint32_t* dst = static_cast<uint32_t*>(args.c) +
                      (static_cast<size_t>(c * args.blocks + blk) * M + row) * N;
      const uint32_t t_row = tbase + ((32u * warp) << 16) + static_cast<uint32_t>((g - g0) * N);
      for (int j = 0; j < N / 32; ++j) {
        uint32_t r[32];
        tmem_ld_32cols(t_row + 32 * j, r);
        tmem_wait_ld();
        if (live) {
          uint4* out = reinterpret_cast<uint4*>(dst + 32 * j);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            out[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, static_cast<uint32_t>(args.tmem_cols));
  }
}

// ---------------------------------------------------------------- host side
using KernelFn = void (*)(CUtensorMap, CUtensorMap, TcArgs);

// (KSTEPS, PANEL) pairs: K bytes per row of 32, 64, 128, 256, 512 and 1024.
template <int KIND>
KernelFn kernel_for_steps(int ksteps) {
  switch (ksteps) {
    case 1: return tc_peak_kernel<KIND, 1, 32>;
    case 2: return tc_peak_kernel<KIND, 2, 64>;
    case 4: return tc_peak_kernel<KIND, 4, 128>;
    case 8: return tc_peak_kernel<KIND, 8, 128>;
    case 16: return tc_peak_kernel<KIND, 16, 128>;
    case 32: return tc_peak_kernel<KIND, 32, 128>;
  }
  return nullptr;
}

KernelFn kernel_for(int kind, int ksteps) {
  switch (kind) {
    case kF16: return kernel_for_steps<kF16>(ksteps);
    case kBF16: return kernel_for_steps<kBF16>(ksteps);
    case kTF32: return kernel_for_steps<kTF32>(ksteps);
    case kI8: return kernel_for_steps<kI8>(ksteps);
    case kE4M3: return kernel_for_steps<kE4M3>(ksteps);
    case kMXF4: return kernel_for_steps<kMXF4>(ksteps);
  }
  return nullptr;
}

int steps_index(int ksteps) {
  switch (ksteps) {
    case 1: return 0;
    case 2: return 1;
    case 4: return 2;
    case 8: return 3;
    case 16: return 4;
    case 32: return 5;
  }
  return -1;
}

const char* instruction_for(int kind) {
  switch (kind) {
    case kF16:
      return "tcgen05.mma.cta_group::1.kind::f16 (f16 x f16 -> f32)";
    case kBF16:
      return "tcgen05.mma.cta_group::1.kind::f16 (bf16 x bf16 -> f32)";
    case kTF32:
      return "tcgen05.mma.cta_group::1.kind::tf32 (tf32 x tf32 -> f32)";
    case kI8:
      return "tcgen05.mma.cta_group::1.kind::i8 (s8 x s8 -> s32)";
    case kE4M3:
      return "tcgen05.mma.cta_group::1.kind::f8f6f4 (e4m3 x e4m3 -> f32)";
    case kMXF4:
      return "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 (e2m1 x e2m1, ue8m0 -> f32)";
  }
  return "";
}

int kind_for(int dtype) {
  switch (dtype) {
    case TCB_T_FP16:
      return kF16;
    case TCB_T_BF16:
      return kBF16;
    case TCB_T_TF32:
      return kTF32;
    case TCB_T_INT8:
      return kI8;
    case TCB_T_FP8E4M3:
      return kE4M3;
    case TCB_T_MXF4:
      return kMXF4;
  }
  return -1;
}

int elem_bits(int kind) {
  switch (kind) {
    case kF16:
    case kBF16:
      return 16;
    case kTF32:
      return 32;
    case kI8:
    case kE4M3:
      return 8;
    case kMXF4:
      return 4;
  }
  return 0;
}

// Instruction descriptor (M = 128 or 64, K-major A and B, dense).
uint32_t make_idesc(int kind, int n, int m) {
  uint32_t d = 0;
  d |= static_cast<uint32_t>(n >> 3) << 17;
  d |= static_cast<uint32_t>(m >> 4) << 24;
  if (kind == kMXF4) {
    d |= 1u << 7;   // A: E2M1
    d |= 1u << 10;  // B: E2M1
    d |= 1u << 23;  // scales: UE8M0
    return d;
  }
  uint32_t c_fmt = 1, ab = 0;
  switch (kind) {
    case kF16:
      ab = 0;
      break;
    case kBF16:
      ab = 1;
      break;
    case kTF32:
      ab = 2;
      break;
    case kI8:
      c_fmt = 2;
      ab = 1;
      break;
    case kE4M3:
      ab = 0;
      break;
  }
  d |= c_fmt << 4;
  d |= ab << 7;
  d |= ab << 10;
  return d;
}

struct Plan {
  int kind = -1;
  int kbytes = 0, panel = 0, halves = 0, ksteps = 0, groups = 0, groups_per_pass = 0;
  int tmem_cols = 0, sf_cols = 0, smem_bytes = 0, smem_request = 0, mma_m = 128;
  uint32_t layout = 0;
  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE;
};

int make_plan(int dtype, int tile_m, int tile_n, int tile_k, int chains, int bps,
              int max_smem_optin, Plan* plan) {
  Plan p;
  p.kind = kind_for(dtype);
  if (p.kind < 0) return TCB_ERR_UNSUPPORTED;
  // 64-row tiles run one M=64 MMA; MX FP4 keeps M = 128 (its scale-factor
  // layout in tensor memory follows M).
  const bool m64 = tile_m == 64 && p.kind != kMXF4;
  if (tile_m != 128 && tile_m != 256 && !m64) return TCB_ERR_UNSUPPORTED;
  if (tile_n < 32 || tile_n > 256 || tile_n % 32) return TCB_ERR_UNSUPPORTED;
  if (chains < 1 || chains > 2) return TCB_ERR_INVALID_ARGUMENT;
  if (bps != 1 && bps != 2 && bps != 4 && bps != 8 && bps != 16) return TCB_ERR_INVALID_ARGUMENT;
  if (tile_k <= 0) return TCB_ERR_INVALID_ARGUMENT;
  const long long kbits = static_cast<long long>(tile_k) * elem_bits(p.kind);
  if (kbits % 8) return TCB_ERR_INVALID_ARGUMENT;
  p.kbytes = static_cast<int>(kbits / 8);
  if (p.kind == kMXF4 && tile_k % 64) return TCB_ERR_INVALID_ARGUMENT;
  if (p.kbytes == 32 || p.kbytes == 64 || p.kbytes == 128) {
    p.panel = p.kbytes;
  } else if (p.kbytes > 128 && p.kbytes % 128 == 0 && p.kbytes <= 1024) {
    p.panel = 128;
  } else {
    return TCB_ERR_UNSUPPORTED;
  }
  p.layout = p.panel == 128 ? 2u : p.panel == 64 ? 4u : 6u;
  p.swizzle = p.panel == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
              : p.panel == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                              : CU_TENSOR_MAP_SWIZZLE_32B;
  p.mma_m = m64 ? 64 : 128;
  p.halves = m64 ? 1 : tile_m / 128;
  p.ksteps = p.kbytes / kMmaKBytes;
  p.groups = p.halves * chains;
  p.tmem_cols = 512 / bps;
  p.sf_cols = p.kind == kMXF4 ? p.ksteps * (4 * p.halves + tile_n / 32) : 0;
  const int acc_cols = p.tmem_cols - p.sf_cols;
  if (acc_cols < tile_n) return TCB_ERR_RESOURCE;
  p.groups_per_pass = acc_cols / tile_n;
  if (p.groups_per_pass > p.groups) p.groups_per_pass = p.groups;
  if (p.groups_per_pass > kMaxGroups) p.groups_per_pass = kMaxGroups;
  p.smem_bytes = (tile_m + chains * tile_n) * p.kbytes + 1024;
  const int floor_bytes = kSmemPerSM / (bps + 1) + 1;
  p.smem_request = p.smem_bytes > floor_bytes ? p.smem_bytes : floor_bytes;
  if (p.smem_bytes > max_smem_optin) return TCB_ERR_RESOURCE;
  if (p.smem_request > max_smem_optin) p.smem_request = max_smem_optin;
  *plan = p;
  return TCB_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  // Resolved once (thread-safe static initialisation).
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    clear_stale_error();
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// 2-D byte view [rows][row_bytes] with a box of [box_rows][panel] bytes.
int make_map(CUtensorMap* map, const void* base, long long rows, int row_bytes, int box_rows,
             int panel, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr) return TCB_ERR_DEVICE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(panel), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TCB_OK : TCB_ERR_INVALID_ARGUMENT;
}

}  // namespace

int tc_tensor_peak(int dtype, const void* A, const void* B, const void* SA, const void* SB,
                   void* C, int blocks, int bps, int tile_m, int tile_n, int tile_k, int chains,
                   int iterations, int* status_dev, cudaStream_t stream) {
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  if (facts.major != 10) return TCB_ERR_UNSUPPORTED;
  Plan p;
  rc = make_plan(dtype, tile_m, tile_n, tile_k, chains, bps, facts.max_smem_optin, &p);
  if (rc != TCB_OK) return rc;
  if (A == nullptr || B == nullptr || C == nullptr || blocks <= 0 || iterations < 1)
    return TCB_ERR_INVALID_ARGUMENT;
  if (p.kind == kMXF4 && (SA == nullptr || SB == nullptr)) return TCB_ERR_INVALID_ARGUMENT;
  if (!aligned(A, 16) || !aligned(B, 16) || !aligned(C, 16)) return TCB_ERR_ALIGNMENT;
  CUtensorMap map_a, map_b;
  rc = make_map(&map_a, A, static_cast<long long>(blocks) * tile_m, p.kbytes, tile_m, p.panel,
                p.swizzle);
  if (rc != TCB_OK) return rc;
  rc = make_map(&map_b, B, static_cast<long long>(chains) * blocks * tile_n, p.kbytes, tile_n,
                p.panel, p.swizzle);
  if (rc != TCB_OK) return rc;
  TcArgs args;
  args.sa = static_cast<const uint8_t*>(SA);
  args.sb = static_cast<const uint8_t*>(SB);
  args.c = C;
  args.status = status_dev;
  args.blocks = blocks;
  args.tile_m = tile_m;
  args.tile_n = tile_n;
  args.kbytes = p.kbytes;
  args.panel = p.panel;
  args.chains = chains;
  args.iterations = iterations;
  args.halves = p.halves;
  args.ksteps = p.ksteps;
  args.groups = p.groups;
  args.groups_per_pass = p.groups_per_pass;
  args.tmem_cols = p.tmem_cols;
  args.sf_groups = p.ksteps * 2;
  args.layout = p.layout;
  args.mma_m = p.mma_m;
  args.idesc = make_idesc(p.kind, tile_n, p.mma_m);
  KernelFn fn = kernel_for(p.kind, p.ksteps);
  if (fn == nullptr) return TCB_ERR_UNSUPPORTED;
  // Raise the dynamic shared-memory cap once per (kernel, device).
  static DeviceIntCache cap_cache[6][6];
  const int cap = cap_cache[p.kind][steps_index(p.ksteps)].get(facts.device, [&] {
    return raise_dynamic_smem(reinterpret_cast<const void*>(fn), facts.max_smem_optin);
  });
  if (cap < 0 || p.smem_bytes > cap) return TCB_ERR_RESOURCE;
  if (p.smem_request > cap) p.smem_request = cap;
  clear_stale_error();
  fn<<<blocks, kThreads, p.smem_request, stream>>>(map_a, map_b, args);
  return launch_status();
}

int tc_kernel_info(int dtype, int tile_m, int tile_n, int tile_k, int chains, int bps,
                   tcb_kernel_info_t* out) {
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  Plan p;
  rc = make_plan(dtype, tile_m, tile_n, tile_k, chains, bps, facts.max_smem_optin, &p);
  if (rc != TCB_OK) return rc;
  cudaFuncAttributes attr;
  KernelFn fn = kernel_for(p.kind, p.ksteps);
  if (fn == nullptr) return TCB_ERR_UNSUPPORTED;
  if (cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(fn)) != cudaSuccess)
    return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = p.smem_request;
  out->threads_per_block = kThreads;
  out->tensor_core = 1;
  copy_str(out->instruction, sizeof(out->instruction), instruction_for(p.kind));
  copy_str(out->execution_kind, sizeof(out->execution_kind), "tensor");
  return TCB_OK;
}

}  // namespace tcb
