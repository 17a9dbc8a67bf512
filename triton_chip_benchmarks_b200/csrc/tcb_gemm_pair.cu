// MX FP4 GEMM on CTA pairs (tcgen05 cta_group::2, sm_100a): C = A . B^T.
//
// Two CTAs of a cluster (one per SM of a TPC) compute one 256 x 256 output
// tile together.  Each CTA loads only its half of the operands -- 128 rows of
// A and 128 rows of B -- and the pair MMA (tcgen05.mma.cta_group::2, M = 256,
// N = 256, issued by the leader CTA) reads both CTAs' shared memory.
//
// Feeding the tensor cores.  At the MX FP4 rate one SM consumes 32 KB of
// operands per 512 cycles.  Measured on B200 (a loads-only TMA probe, one CTA
// per SM), what a CTA can pull from L2 depends on how the bytes are asked
// for, not on how many are in flight: stages of 32 KB made of 16 KB boxes
// reach 45-52 B/clk per SM however deep the ring, 64 KB stages of four boxes
// 66-81, and 64 KB stages of two 3-D boxes (two 128-byte K panels per box)
// 85.  So an operand stage here holds two K blocks (256 bytes of K): A and B
// arrive as one 3-D box each (128 rows x 2 panels, 32 KB), in a ring of
// three.  A stage whose K blocks run past the last whole panel (a ragged K)
// loads 2-D boxes instead, whose out-of-bounds columns TMA fills with zeros.
//
// Scales run ahead.  The E8M0 scales of a stage (6 KB: own 128 A rows and all
// 256 B rows, two K blocks) have their own ring of four slots, in shared
// memory and in tensor memory, filled by a loader warp of their own as soon
// as a slot frees.  Moving a stage's scales into tensor memory (tcgen05.st)
// takes about 460 cycles after they land; issued with the operands by the
// operand producer, the MMA waited on them 9-10 % of its time, and a single
// thread issuing five TMA operations per stage (about 100 cycles each) could
// not keep three operand stages in flight.  (Measured on 8192^3: 3.9 to 5.8
// PFLOP/s across these steps; the breakdown is in the design notes.)  Copying
// the scales with tcgen05.cp from the MMA thread instead (six per K block,
// ordered with the MMAs, as the single-CTA kernel does) removes the writer
// warps and their wait, but each copy takes tensor-pipe time: 5.3 against
// 5.9 PFLOP/s here.
//
// The accumulator (128 rows x 256 fp32 columns per CTA) is drained by 16
// epilogue warps that each load their whole 32 x 64 slice into registers and
// release it at once, so the next tile's MMAs start while C is written.  C
// leaves through shared memory and TMA tensor stores: two 4 KB staging
// buffers, each taken in a fixed turn order by the 8 warps of one group; on a
// pair's last tile, when the operand ring is idle, each warp stages its slice
// in the ring and stores it without turns.
// Direct stores of these rows (32 rows x 16 bytes per instruction, or shuffle-
// transposed to whole lines) slowed the scale writers and the MMA issue; TMA
// stores did not.
//
// Tensor memory per CTA: accumulator columns 0-255, then four scale slots of
// 48 columns (per K block: own A rows in 4 columns and all B rows in 8 per
// pair of K steps).
//
// Roles (736 threads per CTA, both CTAs unless noted):
//   warp 0       operand producer: TMA-loads its A and B halves of each stage
//                (waiting empty, completing on the LEADER's loaded, which
//                expects the bytes of both CTAs);
//   warp 1       (leader only) MMA issuer: waits acc_empty, loaded and full,
//                issues four pair MMAs per K block, commits empty and tfree
//                to both CTAs, and acc_full to both CTAs after each tile;
//   warps 2-17   epilogue (see above), arriving on the leader's acc_empty;
//   warps 18-21  scale writers: wait sloaded and tfree, move this CTA's
//                staged scales into their tensor-memory slot (warp w writes
//                lane quarter w % 4), arrive on this CTA's sfree and the
//                leader's full;
//   warp 22      scale loader: bulk-copies each stage's scales into its slot
//                (waiting sfree, completing on this CTA's sloaded).
// Every wait is bounded; a wait that fails raises the abort flag of both
// CTAs, so the pair leaves its loops together.  A cluster barrier follows
// barrier set-up and precedes teardown, so neither CTA exits while its peer
// may still signal its barriers or read its shared memory.
//
// Counterpart in the reference suite: none (FP4 GEMM is refused at
// bench_tensor.py:1406-1407); same contract as the single-CTA tcb_gemm path.
#include <cudaTypedefs.h>

#include "tcb_device.cuh"
#include "tcb_gemm_common.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

namespace {

using namespace gemm_detail;

constexpr int kPairRows = 128;                                 // A rows and B rows per CTA
constexpr int kPairPanels = 2;                                 // 128-byte K blocks per stage
constexpr int kPairPanelBytes = kPairRows * kBlockBytes;       // 16 KB
constexpr int kPairStageA = kPairPanels * kPairPanelBytes;     // 32 KB
constexpr int kPairStageBytes = 2 * kPairStageA;               // A and B halves, 64 KB
constexpr int kPairStages = 3;
constexpr int kPairScaleBlock = (kPairRows + kTileN) * 8;      // own A + all B scales, one K block
constexpr int kPairSlotBytes = kPairPanels * kPairScaleBlock;  // 6 KB
constexpr int kPairSlots = 4;
constexpr int kPairEpiWarps = 16;
// Back-off of the waits off the critical path (epilogue, scale writers,
// staging turns), in ns, so that 20 warps polling do not take issue slots
// from the producer and MMA warps (measured neutral at 0-256 ns).
constexpr unsigned kPairIdleSleepNs = 64;
constexpr unsigned kPairTurnSleepNs = 128;
constexpr int kPairEpiCols = kTileN / (kPairEpiWarps / 4);     // 64 columns per epilogue warp
constexpr int kPairEpiGroups = 2;
constexpr int kPairEpiGroupWarps = kPairEpiWarps / kPairEpiGroups;
constexpr int kPairScaleWarps = 4;
constexpr int kPairLoaderWarp = 2 + kPairEpiWarps + kPairScaleWarps;  // scale loader
constexpr int kPairThreads = (kPairLoaderWarp + 1) * 32;
constexpr int kPairSlotOffset = kPairStages * kPairStageBytes;
constexpr int kPairStagingOffset = kPairSlotOffset + kPairSlots * kPairSlotBytes;
constexpr int kPairSmem = kPairStagingOffset + kPairEpiGroups * kEpiChunkBytes + 1024;
constexpr int kPairSfCols = kPairPanels * kSfStageCols;        // tensor-memory columns per slot
static_assert(kAccCols + kPairSlots * kPairSfCols <= kTmemCols, "tensor memory overflow");
static_assert(kPairSmem <= 227 * 1024 - 256, "shared memory overflow");
static_assert(kPairSlotOffset % 1024 == 0 && kPairStagingOffset % 1024 == 0,
              "operand stages and staging buffers keep the 1024-byte swizzle alignment");
static_assert(kPairEpiCols == 64, "an epilogue warp drains two 32-column loads");
static_assert(kPairEpiWarps * 2 * kEpiChunkBytes <= kPairStages * kPairStageBytes,
              "the last tile's C slices fit in the operand ring");

struct PairArgs {
  const uint8_t* sa;  // packed E8M0 scales of A (tcb_mx_scales_pack layout)
  const uint8_t* sb;  // packed E8M0 scales of B
  uint32_t* c;        // [M][N] fp32
  int* status;
  int m, n;
  int tiles_m, tiles_n;
  int kblocks;      // 128-byte K blocks (the last may be ragged)
  int full_panels;  // whole 128-byte K blocks reachable through the 3-D maps (0: none)
  int vec_store;    // C rows are 16-byte aligned
  int tma_store;    // C is written through the C tensor map (requires vec_store)
  uint32_t idesc;
};

__device__ __forceinline__ void pair_mma_mxf4(uint32_t d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate, uint32_t tsfa,
                                              uint32_t tsfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], "
      "p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
}

// Walks this pair's stages in order (its tiles t = pair, pair + pairs, ...,
// each in stage_blocks stages of two K blocks).  Advancing is an increment;
// the tile's coordinates are recomputed once per tile.  (A single thread
// recomputing them from a stage index with runtime divisions every stage
// kept the producer too busy to issue loads on time: 44 % of the MMA
// thread's time went to waiting for operands.)
struct PairCursor {
  int t, sb, tm, tn, kb0, nkb;

  __device__ __forceinline__ void start(int first, const PairArgs& a) {
    t = first;
    sb = 0;
    tile_coords(t, a.tiles_m, a.tiles_n, &tm, &tn);
    kb0 = 0;
    nkb = min(kPairPanels, a.kblocks);
  }

  __device__ __forceinline__ void next(int pairs, int stage_blocks, int tiles, const PairArgs& a) {
    if (++sb == stage_blocks) {
      sb = 0;
      t += pairs;
      if (t < tiles) tile_coords(t, a.tiles_m, a.tiles_n, &tm, &tn);
    }
    kb0 = sb * kPairPanels;
    nkb = min(kPairPanels, a.kblocks - kb0);
  }
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_mxf4_kernel(const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b,
                          const __grid_constant__ CUtensorMap map_a3,
                          const __grid_constant__ CUtensorMap map_b3,
                          const __grid_constant__ CUtensorMap map_c,
                          const __grid_constant__ PairArgs args) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t loaded[kPairStages];   // leader: both operand halves landed
  __shared__ __align__(8) uint64_t empty[kPairStages];    // pair MMAs done with the stage
  __shared__ __align__(8) uint64_t sloaded[kPairSlots];   // this CTA's scales landed
  __shared__ __align__(8) uint64_t sfree[kPairSlots];     // this CTA's writers done with the slot
  __shared__ __align__(8) uint64_t full[kPairSlots];      // leader: both CTAs' scales written
  __shared__ __align__(8) uint64_t tfree[kPairSlots];     // pair MMAs done with the tensor-memory slot
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ __align__(8) uint64_t acc_empty;             // leader: both epilogues drained
  __shared__ __align__(8) uint64_t drained;               // leader: every issued MMA finished
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ volatile int store_turn[kPairEpiGroups];     // next staging turn of each group

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);
  const int tiles = args.tiles_m * args.tiles_n;
  const int stage_blocks = (args.kblocks + kPairPanels - 1) / kPairPanels;
  const int my_tiles = pair < tiles ? (tiles - pair + pairs - 1) / pairs : 0;
  const int my_stages = my_tiles * stage_blocks;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
    if (args.full_panels > 0) {
      prefetch_tensormap(&map_a3);
      prefetch_tensormap(&map_b3);
    }
    if (args.tma_store) prefetch_tensormap(&map_c);
    for (int g = 0; g < kPairEpiGroups; ++g) store_turn[g] = 0;
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&loaded[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kPairSlots; ++s) {
      mbar_init(&sloaded[s], 1);
      mbar_init(&sfree[s], kPairScaleWarps);
      mbar_init(&full[s], 2 * kPairScaleWarps);
      mbar_init(&tfree[s], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty, 2 * kPairEpiWarps);
    mbar_init(&drained, 1);
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
  auto pair_wait = [&](uint64_t* bar, uint32_t parity, unsigned sleep_ns = 0) {
    if (wait_or_abort(bar, parity, &abort_flag, args.status, sleep_ns)) return true;
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
      PairCursor op;
      op.start(pair, args);
      for (int it = 0; it < my_stages && !abort_flag; ++it) {
        const int s = it % kPairStages;
        const uint32_t phase = static_cast<uint32_t>(it / kPairStages) & 1u;
        if (!pair_wait(&empty[s], phase ^ 1u)) break;
        const int arow = op.tm * 2 * kPairRows + static_cast<int>(rank) * kPairRows;
        const int brow = op.tn * kTileN + static_cast<int>(rank) * kPairRows;
        uint8_t* stage = smem + s * kPairStageBytes;
        // Both CTAs' operand bytes complete on the leader's barrier.
        const uint32_t lead_loaded = mapa_shared(smem_addr(&loaded[s]), 0);
        if (rank == 0) mbar_arrive_expect_tx(&loaded[s], 2 * 2 * op.nkb * kPairPanelBytes);
        if (op.nkb == kPairPanels && op.kb0 + kPairPanels <= args.full_panels) {
          tma_load_3d_pair(stage, &map_a3, 0, arow, op.kb0, lead_loaded);
          tma_load_3d_pair(stage + kPairStageA, &map_b3, 0, brow, op.kb0, lead_loaded);
        } else {
          for (int q = 0; q < op.nkb; ++q) {
            const int x = (op.kb0 + q) * kBlockBytes;
            tma_load_2d_pair(stage + q * kPairPanelBytes, &map_a, x, arow, lead_loaded);
            tma_load_2d_pair(stage + kPairStageA + q * kPairPanelBytes, &map_b, x, brow,
                             lead_loaded);
          }
        }
        op.next(pairs, stage_blocks, tiles, args);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && rank == 0) {
      const uint64_t desc_const = smem_desc(0, 16, 8 * kBlockBytes, 2u);
      const uint32_t smem0 = smem_addr(smem) >> 4;
      int it = 0;
      for (int ti = 0; ti < my_tiles && !abort_flag; ++ti) {
        if (!pair_wait(&acc_empty, (static_cast<uint32_t>(ti) & 1u) ^ 1u)) break;
        tc_fence_after();
        for (int sb = 0; sb < stage_blocks; ++sb, ++it) {
          const int s = it % kPairStages;
          const int slot = it % kPairSlots;
          if (!pair_wait(&loaded[s], static_cast<uint32_t>(it / kPairStages) & 1u)) break;
          if (!pair_wait(&full[slot], static_cast<uint32_t>(it / kPairSlots) & 1u)) break;
          tc_fence_after();
          const int nkb = min(kPairPanels, args.kblocks - sb * kPairPanels);
          const uint32_t a_lo = smem0 + static_cast<uint32_t>(s * kPairStageBytes >> 4);
          const uint32_t b_lo = a_lo + (kPairStageA >> 4);
          const uint32_t sf = tbase + kAccCols + static_cast<uint32_t>(slot * kPairSfCols);
#pragma unroll
          for (int q = 0; q < kPairPanels; ++q) {
            if (q >= nkb) break;
            const uint32_t panel = static_cast<uint32_t>(q * (kPairPanelBytes >> 4));
            const uint32_t sfq = sf + static_cast<uint32_t>(q * kSfStageCols);
#pragma unroll
            for (int k = 0; k < kStepsPerBlock; ++k) {
              pair_mma_mxf4(tbase, desc_const | (a_lo + panel + static_cast<uint32_t>(k * 2)),
                            desc_const | (b_lo + panel + static_cast<uint32_t>(k * 2)),
                            sf_idesc(args.idesc, k), (sb | q | k) != 0, sf_cols_a(sfq, k),
                            sf_cols_b(sfq, k));
            }
          }
          tc_commit_pair(&empty[s], 0x3);
          tc_commit_pair(&tfree[slot], 0x3);
        }
        if (abort_flag) break;
        tc_commit_pair(&acc_full, 0x3);
      }
      // Nothing this thread issued may still run when the pair tears down.
      tc_commit_pair(&drained, 0x1);
      if (!mbar_wait(&drained, 0)) report_status(args.status, TCB_ERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp < 2 + kPairEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // Tensor-memory lanes 32(warp % 4).. are this warp's rows; its columns are
    // one 64-wide slice.  The whole slice comes into registers before the
    // accumulator is released.  C then goes out through the group's staging
    // buffer in a fixed turn order (turn = tile x 8 + slot): stage 32 columns,
    // TMA-store them, wait until the store has read the buffer, repeat, and
    // hand the buffer on.
    const int quarter = warp & 3;
    const int col0 = ((warp - 2) >> 2) * kPairEpiCols;
    const int group = (warp - 2) / kPairEpiGroupWarps;
    const int slot = (warp - 2) % kPairEpiGroupWarps;
    uint8_t* staging = smem + kPairStagingOffset + group * kEpiChunkBytes;
    const uint32_t lead_acc_empty = mapa_shared(smem_addr(&acc_empty), 0);
    const uint32_t taddr = tbase + ((32u * quarter) << 16) + static_cast<uint32_t>(col0);
    // Bounded wait for this warp's staging turn.
    auto turn_wait = [&](int mine) {
      if (store_turn[group] == mine) return true;
      const unsigned long long start = globaltimer_ns();
      while (store_turn[group] != mine) {
        __nanosleep(kPairTurnSleepNs);
        if (abort_flag) return false;
        if (globaltimer_ns() - start > kWaitTimeoutNs) {
          abort_flag = 1;
          st_shared_cluster_u32(peer_abort, 1u);
          report_status(args.status, TCB_ERR_TIMEOUT);
          return false;
        }
      }
      return true;
    };
    for (int ti = 0; ti < my_tiles; ++ti) {
      // Warp-uniform exits: tcgen05.ld and .st need the whole warp.
      if (!__all_sync(0xffffffffu, pair_wait(&acc_full, static_cast<uint32_t>(ti) & 1u,
                                              kPairIdleSleepNs)))
        break;
      tc_fence_after();
      uint32_t r[2][32];
      acc_load<2>(taddr, r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty);
      int tm, tn;
      tile_coords(pair + ti * pairs, args.tiles_m, args.tiles_n, &tm, &tn);
      const int row0 = tm * 2 * kPairRows + static_cast<int>(rank) * kPairRows + 32 * quarter;
      const int c = tn * kTileN + col0;
      if (args.tma_store && ti + 1 == my_tiles) {
        // Last tile: every MMA has finished reading the operand ring (acc_full
        // follows their completion) and no load refills it, so each warp
        // stages its whole slice in 8 KB of the ring of its own and stores it
        // at once instead of waiting for staging turns (with one or two tiles
        // per pair the turns were the critical path).
        uint8_t* own = smem + (warp - 2) * 2 * kEpiChunkBytes;
#pragma unroll
        for (int q = 0; q < 2; ++q) stage_chunk(own + q * kEpiChunkBytes, lane, r[q]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int q = 0; q < 2; ++q)
            tma_store_2d(&map_c, c + 32 * q, row0, own + q * kEpiChunkBytes);
          bulk_commit_group();
        }
        __syncwarp();
      } else if (args.tma_store) {
        const int mine = ti * kPairEpiGroupWarps + slot;
        if (!__all_sync(0xffffffffu, turn_wait(mine))) break;
        __threadfence_block();
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          stage_chunk(staging, lane, r[q]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_c, c + 32 * q, row0, staging);
            bulk_commit_group();
            bulk_wait_group_read<0>();
          }
          __syncwarp();
        }
        if (lane == 0) store_turn[group] = mine + 1;
      } else if (row0 + lane < args.m) {
        acc_store<2>(args.c + static_cast<size_t>(row0 + lane) * args.n + c, r, c, args.n,
                     args.vec_store);
      }
    }
    if (lane == 0) bulk_wait_group_all();  // C stores complete before the CTA retires
  } else if (warp < kPairLoaderWarp) {
    // ------------------------------------------------------ scale writers
    // Lane l writes rows 32j+l of each staged K block's scales into this
    // CTA's tensor-memory slot (two K steps per word).
    const int quarter = warp & 3;
    const uint32_t lane_base = tbase + ((32u * quarter) << 16) + kAccCols;
    int sb = 0;  // stage block of `it` within its tile
    for (int it = 0; it < my_stages; ++it) {
      const int slot = it % kPairSlots;
      // Warp-uniform exit: tcgen05.st needs the whole warp.  The stage's
      // scales have landed, and the MMAs that read the tensor-memory slot's
      // previous contents (kPairSlots stages back) have finished.
      const uint32_t round = static_cast<uint32_t>(it / kPairSlots) & 1u;
      if (!__all_sync(0xffffffffu, pair_wait(&sloaded[slot], round, kPairIdleSleepNs) &&
                                       pair_wait(&tfree[slot], round ^ 1u, kPairIdleSleepNs)))
        break;
      const int nkb = min(kPairPanels, args.kblocks - sb * kPairPanels);
      if (++sb == stage_blocks) sb = 0;
      // Packed layout: lane l's 16 bytes of each 512-byte half are exactly its
      // words for the four A columns (rows l, 32+l, 64+l, 96+l), and those of
      // B rows 0-127 and 128-255 for the eight B columns.
      const uint8_t* ss = smem + kPairSlotOffset + slot * kPairSlotBytes + lane * 16;
#pragma unroll
      for (int q = 0; q < kPairPanels; ++q) {
        if (q >= nkb) break;
        const uint8_t* h = ss + q * 1024;
        write_scale_block(lane_base + static_cast<uint32_t>(slot * kPairSfCols + q * kSfStageCols),
                          h, h + kPairPanels * 1024, h + 2 * kPairPanels * 1024);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sfree[slot]);  // the shared-memory slot may be refilled
        mbar_arrive_cluster(mapa_shared(smem_addr(&full[slot]), 0));
      }
    }
  } else if (lane == 0) {
    // -------------------------------------------------------- scale loader
    // Scales of each stage into slot j % kPairSlots as soon as this CTA's
    // writers have moved the slot's previous stage into tensor memory (not
    // when its MMAs finish, which would leave the loads only about three
    // stages of lead): [A own rows][B rows 0-127][B rows 128-255], nkb KiB
    // each (consecutive K blocks of a row block are contiguous in the packed
    // layout).  Its own warp, so neither the operand producer nor the scale
    // writers wait for these copies to be issued.
    const size_t rb_bytes = static_cast<size_t>(args.kblocks) * 1024;
    PairCursor sc;
    sc.start(pair, args);
    for (int j = 0; j < my_stages && !abort_flag; ++j) {
      const int slot = j % kPairSlots;
      if (!pair_wait(&sfree[slot], (static_cast<uint32_t>(j / kPairSlots) & 1u) ^ 1u)) break;
      uint8_t* ss = smem + kPairSlotOffset + slot * kPairSlotBytes;
      const uint32_t sbytes = static_cast<uint32_t>(sc.nkb) * 1024;
      mbar_arrive_expect_tx(&sloaded[slot], 3 * sbytes);
      bulk_load_1d(ss, args.sa + (2 * sc.tm + rank) * rb_bytes + sc.kb0 * 1024, sbytes,
                   &sloaded[slot]);
      bulk_load_1d(ss + kPairPanels * 1024, args.sb + (2 * sc.tn) * rb_bytes + sc.kb0 * 1024,
                   sbytes, &sloaded[slot]);
      bulk_load_1d(ss + 2 * kPairPanels * 1024, args.sb + (2 * sc.tn + 1) * rb_bytes + sc.kb0 * 1024,
                   sbytes, &sloaded[slot]);
      sc.next(pairs, stage_blocks, tiles, args);
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

// A [rows][row_bytes] as 128-byte x 128-row boxes (2-D) and, when it has at
// least two whole 128-byte K blocks, as 128-byte x 128-row x 2-block boxes
// over the whole K blocks (3-D: x in the block, y the row, z the block).
// `*full_panels` is set to 0 when no 3-D map is made (then every stage loads
// 2-D boxes).
int pair_maps(CUtensorMap* map2, CUtensorMap* map3, const void* base, long long rows,
              long long row_bytes, int* full_panels) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return TCB_ERR_DEVICE;
  void* p = const_cast<void*>(base);
  cuuint64_t dims2[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides2[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box2[2] = {static_cast<cuuint32_t>(kBlockBytes), static_cast<cuuint32_t>(kPairRows)};
  cuuint32_t estr[3] = {1, 1, 1};
  if (fn(map2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p, dims2, strides2, box2, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return TCB_ERR_INVALID_ARGUMENT;
  *map3 = CUtensorMap{};
  if (*full_panels < kPairPanels) {
    *full_panels = 0;
    return TCB_OK;
  }
  cuuint64_t dims3[3] = {static_cast<cuuint64_t>(kBlockBytes), static_cast<cuuint64_t>(rows),
                         static_cast<cuuint64_t>(*full_panels)};
  cuuint64_t strides3[2] = {static_cast<cuuint64_t>(row_bytes),
                            static_cast<cuuint64_t>(kBlockBytes)};
  cuuint32_t box3[3] = {static_cast<cuuint32_t>(kBlockBytes), static_cast<cuuint32_t>(kPairRows),
                        static_cast<cuuint32_t>(kPairPanels)};
  if (fn(map3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, p, dims3, strides3, box3, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    *map3 = CUtensorMap{};
    *full_panels = 0;  // the 2-D boxes still cover every stage
  }
  return TCB_OK;
}

// C [rows][cols] fp32 as 32 x 32 boxes in the SWIZZLE_128B layout the
// epilogue stages (16-byte row pitch and base required).
int pair_map_c(CUtensorMap* map, void* base, int rows, int cols) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return TCB_ERR_DEVICE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? TCB_OK
             : TCB_ERR_INVALID_ARGUMENT;
}

}  // namespace

// MX FP4 GEMM on CTA pairs for M > 128: tensor maps, arguments and launch of
// `blocks / 2` persistent pairs (all the pairs that fit at once by default).
int gemm_pair_run(const void* A, const void* B, const void* SA, const void* SB, void* C, int M,
                  int N, int K, int blocks, int* status, uint32_t idesc, const DeviceFacts& facts,
                  cudaStream_t stream) {
  const long long kbytes = static_cast<long long>(K) / 2;
  PairArgs args;
  args.sa = static_cast<const uint8_t*>(SA);
  args.sb = static_cast<const uint8_t*>(SB);
  args.c = static_cast<uint32_t*>(C);
  args.status = status;
  args.m = M;
  args.n = N;
  args.tiles_m = (M + 2 * kPairRows - 1) / (2 * kPairRows);
  args.tiles_n = (N + kTileN - 1) / kTileN;
  args.kblocks = static_cast<int>((kbytes + kBlockBytes - 1) / kBlockBytes);
  args.vec_store = N % 4 == 0 && aligned(C, 16);
  args.idesc = idesc;
  CUtensorMap map_a, map_b, map_a3, map_b3;
  int panels_a = static_cast<int>(kbytes / kBlockBytes), panels_b = panels_a;
  int rc;
  if ((rc = pair_maps(&map_a, &map_a3, A, M, kbytes, &panels_a)) != TCB_OK) return rc;
  if ((rc = pair_maps(&map_b, &map_b3, B, N, kbytes, &panels_b)) != TCB_OK) return rc;
  args.full_panels = panels_a < panels_b ? panels_a : panels_b;
  CUtensorMap map_c{};
  args.tma_store = args.vec_store && pair_map_c(&map_c, C, M, N) == TCB_OK;
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
  const int tiles = args.tiles_m * args.tiles_n;
  int pairs = blocks > 0 ? blocks / 2 : facts.sm_count / 2;
  if (pairs < 1) pairs = 1;
  if (pairs > tiles) pairs = tiles;
  if (pairs > resident) pairs = resident;
  clear_stale_error();
  gemm_pair_mxf4_kernel<<<2 * pairs, kPairThreads, kPairSmem, stream>>>(map_a, map_b, map_a3,
                                                                          map_b3, map_c, args);
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
