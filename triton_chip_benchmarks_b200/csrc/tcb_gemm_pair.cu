// MX FP4 GEMM on CTA pairs (tcgen05 cta_group::2, sm_100a): C = A . B^T.
//
// Two CTAs of a cluster (one per SM of a TPC) compute one 256 x 256 output
// tile together.  Each CTA loads only its half of the operands -- 128 rows of
// A and 128 rows of B per 128-byte K block -- and the pair MMA
// (tcgen05.mma.cta_group::2, M = 256, N = 256, issued by the leader CTA)
// reads both CTAs' shared memory.  Per SM that is 32 KB of operands per 512
// MMA cycles instead of 48 KB for a single-CTA 128 x 256 tile: a third less
// L2 -> SM traffic, which is what bounds the single-CTA MX FP4 GEMM.
//
// Each CTA's tensor memory holds its 128 rows x 256 columns fp32 accumulator
// plus a ring of E8M0 scale slots: its own 128 A rows (4 columns per K step)
// and all 256 B rows (8 columns per K step).
//
// Roles (320 threads per CTA, both CTAs unless noted):
//   warp 0      producer: waits empty[s] (its own; the leader's commit arrives
//               on both CTAs), TMA-loads its A and B halves completing on the
//               LEADER's loaded[s] (the leader posts the byte count of both
//               halves), and bulk-copies its scales completing on its own
//               sloaded[s];
//   warp 1      (leader only) MMA issuer: waits acc_empty, loaded[s] and
//               full[s], issues four pair MMAs per K block, commits empty[s]
//               to both CTAs, and acc_full to both CTAs after each tile;
//   warps 2-5   epilogue: drain this CTA's accumulator lanes in two
//               128-column round trips, arrive on the leader's acc_empty once
//               the last columns are in registers, and write C through
//               swizzled shared staging and TMA tensor stores;
//   warps 6-9   scale writers: move this CTA's staged scales into its scale
//               slot and arrive on the leader's full[s].
// Every wait is bounded; a wait that fails raises the abort flag of both
// CTAs, so the pair leaves its loops together.  A cluster barrier follows barrier set-up and
// precedes teardown, so neither CTA exits while its peer may still signal its
// barriers or read its shared memory.
//
// Counterpart in the reference suite: none (FP4 GEMM is refused at
// bench_tensor.py:1406-1407); same contract as the single-CTA tcb_gemm path.
#include <cudaTypedefs.h>

#include "tcb_device.cuh"
#include "tcb_gemm_common.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

using namespace gemm_detail;

constexpr int kPairRows = 128;                                // A rows and B rows per CTA
constexpr int kPairStageA = kPairRows * kBlockBytes;          // 16 KB
constexpr int kPairStageB = kPairRows * kBlockBytes;          // 16 KB
constexpr int kPairStageS = (kPairRows + kTileN) * 8;         // own A scales + all B scales
constexpr int kPairStageBytes = kPairStageA + kPairStageB + kPairStageS;
constexpr int kPairStages = 5;
constexpr int kPairSmem = kPairStages * kPairStageBytes + kEpiSmem + 1024;
constexpr int kPairThreads = (6 + kScaleWarps) * 32;
static_assert(kAccCols + kPairStages * kSfStageCols <= kTmemCols, "tensor memory overflow");
static_assert(kPairSmem <= 227 * 1024, "shared memory overflow");
static_assert(kPairStageBytes % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");

__device__ __forceinline__ void pair_mma_mxf4(uint32_t d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate, uint32_t tsfa,
                                              uint32_t tsfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], "
      "p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_mxf4_kernel(const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b,
                          const __grid_constant__ CUtensorMap map_c, const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t loaded[kPairStages];   // leader: both operand halves landed
  __shared__ __align__(8) uint64_t sloaded[kPairStages];  // this CTA's scales landed
  __shared__ __align__(8) uint64_t full[kPairStages];     // leader: both CTAs' scales written
  __shared__ __align__(8) uint64_t empty[kPairStages];    // pair MMAs done with the stage
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ __align__(8) uint64_t acc_empty;             // leader: both epilogues drained
  __shared__ __align__(8) uint64_t drained;               // leader: every issued MMA finished
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);
  const int tiles = args.tiles_m * args.tiles_n;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
    if (args.tma_store) prefetch_tensormap(&map_c);
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&loaded[s], 1);
      mbar_init(&sloaded[s], 1);
      mbar_init(&full[s], 2 * kScaleWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty, 2 * kEpilogueWarps);
    mbar_init(&drained, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(&tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated
  tc_fence_after();
  const uint32_t tbase = tmem_slot;
  // An abort on either CTA stops both: a wait that fails also raises the
  // peer's flag (a store into its shared memory, which stays valid until the
  // teardown cluster barrier), so neither CTA sits out a full timeout on
  // barriers the other no longer signals.
  const uint32_t peer_abort = mapa_shared(smem_addr(const_cast<int*>(&abort_flag)), rank ^ 1u);
  auto pair_wait = [&](uint64_t* bar, uint32_t parity) {
    if (wait_or_abort(bar, parity, &abort_flag, args.status)) return true;
    st_shared_cluster_u32(peer_abort, 1u);
    return false;
  };
  if (threadIdx.x == 0 && rank != 0) {
    // The pair MMA addresses both CTAs' tensor memory with the leader's column base.
    if (ld_shared_cluster_u32(mapa_shared(smem_addr(&tmem_slot), 0)) != tbase) {
      abort_flag = 1;
      st_shared_cluster_u32(peer_abort, 1u);
      report_status(args.status, TCB_ERR_DEVICE);
    }
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const size_t rb_bytes = static_cast<size_t>(args.kblocks) * 1024;
      int it = 0;
      for (int t = pair; t < tiles && !abort_flag; t += pairs) {
        int tm, tn;
        tile_coords(t, args.tiles_m, args.tiles_n, &tm, &tn);
        const int arow = tm * 2 * kPairRows + static_cast<int>(rank) * kPairRows;
        const int brow = tn * kTileN + static_cast<int>(rank) * kPairRows;
        for (int kb = 0; kb < args.kblocks; ++kb, ++it) {
          const int s = it % kPairStages;
          const uint32_t phase = static_cast<uint32_t>(it / kPairStages) & 1u;
          if (!pair_wait(&empty[s], phase ^ 1u)) break;
          uint8_t* stage = smem + s * kPairStageBytes;
          const uint32_t lead_loaded = mapa_shared(smem_addr(&loaded[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&loaded[s], 2 * (kPairStageA + kPairStageB));
          tma_load_2d_pair(stage, &map_a, kb * kBlockBytes, arow, lead_loaded);
          tma_load_2d_pair(stage + kPairStageA, &map_b, kb * kBlockBytes, brow, lead_loaded);
          uint8_t* ss = stage + kPairStageA + kPairStageB;
          mbar_arrive_expect_tx(&sloaded[s], kPairStageS);
          bulk_load_1d(ss, args.sa + (2 * tm + rank) * rb_bytes + kb * 1024, 1024, &sloaded[s]);
          bulk_load_1d(ss + 1024, args.sb + (2 * tn) * rb_bytes + kb * 1024, 1024, &sloaded[s]);
          bulk_load_1d(ss + 2048, args.sb + (2 * tn + 1) * rb_bytes + kb * 1024, 1024,
                       &sloaded[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && rank == 0) {
      const uint64_t desc_const = smem_desc(0, 16, 8 * kBlockBytes, 2u);
      const uint32_t smem0 = smem_addr(smem) >> 4;
      int it = 0, ti = 0;
      for (int t = pair; t < tiles && !abort_flag; t += pairs, ++ti) {
        if (!pair_wait(&acc_empty, (static_cast<uint32_t>(ti) & 1u) ^ 1u)) break;
        tc_fence_after();
        for (int kb = 0; kb < args.kblocks; ++kb, ++it) {
          const int s = it % kPairStages;
          const uint32_t phase = static_cast<uint32_t>(it / kPairStages) & 1u;
          if (!pair_wait(&loaded[s], phase)) break;
          if (!pair_wait(&full[s], phase)) break;
          tc_fence_after();
          const uint32_t a_lo = smem0 + static_cast<uint32_t>(s * kPairStageBytes >> 4);
          const uint32_t b_lo = a_lo + (kPairStageA >> 4);
          const uint32_t sf = tbase + kAccCols + static_cast<uint32_t>(s * kSfStageCols);
#pragma unroll
          for (int k = 0; k < kStepsPerBlock; ++k) {
            pair_mma_mxf4(tbase, desc_const | (a_lo + static_cast<uint32_t>(k * 2)),
                          desc_const | (b_lo + static_cast<uint32_t>(k * 2)),
                          sf_idesc(args.idesc, k), (kb | k) != 0, sf_cols_a(sf, k),
                          sf_cols_b(sf, k));
          }
          tc_commit_pair(&empty[s], 0x3);
        }
        if (abort_flag) break;
        tc_commit_pair(&acc_full, 0x3);
      }
      // Nothing this thread issued may still run when the pair tears down.
      tc_commit_pair(&drained, 0x1);
      if (!mbar_wait(&drained, 0)) report_status(args.status, TCB_ERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp < 2 + kEpilogueWarps) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const uint32_t lead_acc_empty = mapa_shared(smem_addr(&acc_empty), 0);
    uint8_t* epi_stage = smem + kPairStages * kPairStageBytes + (warp - 2) * kEpiWarpBytes;
    int ti = 0, issued = 0;
    for (int t = pair; t < tiles; t += pairs, ++ti) {
      if (!pair_wait(&acc_full, static_cast<uint32_t>(ti) & 1u)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(t, args.tiles_m, args.tiles_n, &tm, &tn);
      const int row0 = tm * 2 * kPairRows + static_cast<int>(rank) * kPairRows + 32 * quarter;
      const uint32_t taddr = tbase + ((32u * quarter) << 16);
      // 64-column round trips; the accumulator is released as soon as its
      // last columns are in registers, so C traffic overlaps the next tile's
      // MMAs.
      uint32_t r[kEpiChunks][32];
      const int row = row0 + lane;
      const bool row_in = row < args.m;
      uint32_t* dst = args.c + static_cast<size_t>(row) * args.n + tn * kTileN;
#pragma unroll 1
      for (int c0 = 0; c0 < kTileN; c0 += 32 * kEpiChunks) {
        acc_load<kEpiChunks>(taddr + c0, r);
        if (c0 + 32 * kEpiChunks == kTileN) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_acc_empty);
        }
        if (args.tma_store)
          acc_tma_store<kEpiChunks>(&map_c, epi_stage, lane, r, tn * kTileN + c0, row0, issued);
        else if (row_in)
          acc_store<kEpiChunks>(dst + c0, r, tn * kTileN + c0, args.n, args.vec_store);
      }
    }
    if (lane == 0) bulk_wait_group_all();  // C stores complete before the CTA retires
  } else {
    // ------------------------------------------------------ scale writers
    // Lane l takes rows 32j+l (8 bytes each) of the staged scales and writes
    // them into this CTA's scale slot for the stage (two K steps per word).
    const int quarter = warp & 3;
    const uint32_t lane_base = tbase + ((32u * quarter) << 16) + kAccCols;
    int it = 0;
    for (int t = pair; t < tiles && !abort_flag; t += pairs) {
      for (int kb = 0; kb < args.kblocks; ++kb, ++it) {
        const int s = it % kPairStages;
        const uint32_t phase = static_cast<uint32_t>(it / kPairStages) & 1u;
        if (!pair_wait(&sloaded[s], phase)) break;
        const uint8_t* ss = smem + s * kPairStageBytes + kPairStageA + kPairStageB + lane * 8;
        uint2 fa[4], fb[kTileN / 32];
#pragma unroll
        for (int j = 0; j < 4; ++j) fa[j] = *reinterpret_cast<const uint2*>(ss + 256 * j);
#pragma unroll
        for (int j = 0; j < kTileN / 32; ++j)
          fb[j] = *reinterpret_cast<const uint2*>(ss + 1024 + 256 * j);
        write_scale_slot(lane_base + static_cast<uint32_t>(s * kSfStageCols), fa, fb);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&full[s]), 0));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the peer may still touch its shared memory
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, kTmemCols);
  }
}

}  // namespace

// Launch the pair kernel: `pairs` clusters of two persistent CTAs.
int gemm_pair_launch(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_c,
                     const GemmArgs& args, int pairs, const DeviceFacts& facts,
                     cudaStream_t stream) {
  static DeviceIntCache cap_cache, resident_cache;
  const int cap = cap_cache.get(facts.device, [&] {
    return raise_dynamic_smem(reinterpret_cast<const void*>(gemm_pair_mxf4_kernel),
                              facts.max_smem_optin);
  });
  if (cap < kPairSmem) return TCB_ERR_RESOURCE;
  // Pairs that can be resident at once: persistent pairs beyond that would
  // only start when others finish, serialising their tiles.
  const int resident = resident_cache.get(facts.device, [&] {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(2 * (facts.sm_count / 2), 1, 1);
    config.blockDim = dim3(kPairThreads, 1, 1);
    config.dynamicSmemBytes = kPairSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_mxf4_kernel, &config) != cudaSuccess ||
        clusters < 1) {
      clear_stale_error();
      clusters = facts.sm_count / 2;
    }
    return clusters;
  });
  if (pairs > resident) pairs = resident;
  clear_stale_error();
  gemm_pair_mxf4_kernel<<<2 * pairs, kPairThreads, kPairSmem, stream>>>(map_a, map_b, map_c,
                                                                          args);
  return launch_status();
}

int gemm_pair_info(tcb_kernel_info_t* out) {
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(gemm_pair_mxf4_kernel)) !=
      cudaSuccess)
    return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = kPairSmem;
  out->threads_per_block = kPairThreads;
  out->tensor_core = 1;
  out->pipeline_stages = kPairStages;
  out->tile_m = 2 * kPairRows;
  out->tile_n = kTileN;
  out->cluster_ctas = 2;
  return TCB_OK;
}

}  // namespace tcb
