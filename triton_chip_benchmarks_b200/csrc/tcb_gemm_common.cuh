// Pieces shared by the tcgen05 GEMM kernels (one CTA per tile, and CTA pairs):
// tile constants, kernel arguments, bounded barrier waits, bulk copies, the
// grouped tile order and streaming stores.
#pragma once

#include <cstdint>

#include "tcb_device.cuh"

namespace tcb {
namespace gemm_detail {

enum GKind : int { gF16 = 0, gBF16 = 1, gTF32 = 2, gI8 = 3, gE4M3 = 4, gMXF4 = 5 };

constexpr int kTileN = 256;
constexpr int kBlockBytes = 128;     // K bytes per pipeline stage (one SWIZZLE_128B panel)
constexpr int kStepsPerBlock = 4;    // 32-byte MMA K steps per block
constexpr int kAccCols = kTileN;     // fp32 accumulator columns per M=128 half
constexpr int kSmemBudget = 227 * 1024 - 1024;

// MX scales in tensor memory: one 32-bit column word holds the scale pairs of
// two consecutive K steps (bytes 0-1 and 2-3), selected per MMA by the scale
// factor ID of the instruction descriptor (0 or 2).  A takes 4 columns and B 8
// columns per pair of K steps.
constexpr int kSfPairCols = 4 + kTileN / 32;
constexpr int kMaxStages = 6;
constexpr int kSfStageCols = (kStepsPerBlock / 2) * kSfPairCols;

// Scale-factor columns and descriptor of K step k of a block whose scale slot
// starts at column `sf`.
__device__ __forceinline__ uint32_t sf_cols_a(uint32_t sf, int k) { return sf + (k >> 1) * kSfPairCols; }
__device__ __forceinline__ uint32_t sf_cols_b(uint32_t sf, int k) {
  return sf + (k >> 1) * kSfPairCols + 4;
}
__device__ __forceinline__ uint32_t sf_idesc(uint32_t idesc, int k) {
  const uint32_t id = 2u * static_cast<uint32_t>(k & 1);
  return idesc | (id << 29) | (id << 4);  // A scale factor ID [29,31), B [4,6)
}

// Scales of one K block into this warp's lane quarter of the tensor-memory
// slot at `lane_col` (tcgen05.st, two K steps per 32-bit word).  `a`, `b0` and
// `b1` point at this lane's 16 bytes (lane x 16) of the 1 KB packed blocks
// (tcb_mx_scales_pack layout) of A's 128 rows and of B rows 0-127 and
// 128-255 in shared memory.  In each 512-byte half (K steps 2kp, 2kp+1) those
// 16 bytes are the lane's words for rows l, 32+l, 64+l, 96+l: A's four
// columns, and B's eight with the second block.
__device__ __forceinline__ void write_scale_block(uint32_t lane_col, const uint8_t* a,
                                                  const uint8_t* b0, const uint8_t* b1) {
#pragma unroll
  for (int kp = 0; kp < 2; ++kp) {
    const uint4 wa = *reinterpret_cast<const uint4*>(a + kp * 512);
    const uint4 w0 = *reinterpret_cast<const uint4*>(b0 + kp * 512);
    const uint4 w1 = *reinterpret_cast<const uint4*>(b1 + kp * 512);
    const uint32_t va[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t vb[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    tmem_st_4cols(lane_col + static_cast<uint32_t>(kp * kSfPairCols), va);
    tmem_st_8cols(lane_col + static_cast<uint32_t>(kp * kSfPairCols) + 4, vb);
  }
}
constexpr int kTmemCols = 512;
constexpr int kEpilogueWarps = 4;
constexpr int kScaleWarps = 4;

struct GemmArgs {
  const uint8_t* sa;  // [M][K/32] E8M0 (MX FP4)
  const uint8_t* sb;  // [N][K/32]
  uint32_t* c;        // [M][N] 32-bit
  int* status;
  int m, n, kbytes, kgroups;  // kgroups = K/32 scale groups per row
  int tiles_m, tiles_n, kblocks;
  int vec_store;  // C rows are 16-byte aligned (N % 4 == 0 and C 16-byte aligned)
  int tma_store;  // C is written through the C tensor map (requires vec_store)
  uint32_t idesc;
};

// Bounded wait on an mbarrier phase.  `sleep_ns` > 0 backs off between polls
// (for roles whose wait is not on the critical path: many warps polling in a
// tight loop take issue slots from the warps that feed the tensor cores).
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, int* status,
                                              unsigned sleep_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (sleep_ns) __nanosleep(sleep_ns);
    if (*abort_flag) return false;
    if (globaltimer_ns() - start > kWaitTimeoutNs) {
      *abort_flag = 1;
      report_status(status, TCB_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Untiled bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, uint32_t size,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(smem_dst)),
      "l"(src), "r"(size), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Tile t -> (tm, tn) in groups of kGroupM row-blocks: the tiles a wave of
// persistent CTAs works on at once share few A row-blocks and B column-blocks,
// so their operands stay in L2.
constexpr int kGroupM = 8;

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int* tm, int* tn) {
  const int per_group = kGroupM * tiles_n;
  const int group = t / per_group;
  const int first = group * kGroupM;
  const int rows = min(tiles_m - first, kGroupM);
  const int r = t - group * per_group;
  *tm = first + r % rows;
  *tn = r / rows;
}

__device__ __forceinline__ void st_stream_u4(void* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// ------------------------------------------------ C through TMA tensor stores
// Each epilogue warp owns two 4 KB staging buffers (32 rows x 32 fp32, the
// SWIZZLE_128B image: 16-byte chunk c of row r at r*128 + ((c ^ (r % 8)) * 16)),
// so a warp's 16-byte shared stores hit all 32 banks.
constexpr int kEpiChunkBytes = 32 * 32 * 4;
constexpr int kEpiWarpBytes = 2 * kEpiChunkBytes;
constexpr int kEpiSmem = 4 * kEpiWarpBytes;  // four epilogue warps
constexpr int kEpiChunks = 2;                 // 32-column chunks per tensor-memory round trip

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y,
                                             const void* smem_src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_addr(smem_src))
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed store groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed store group of this thread has completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// One 32 x 32 chunk (lane = row) into a staging buffer, swizzled.
__device__ __forceinline__ void stage_chunk(uint8_t* buf, int lane, const uint32_t (&v)[32]) {
  uint8_t* row = buf + lane * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(row + ((c ^ (lane & 7)) << 4)) =
        make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// Store CH loaded 32-column chunks of this warp's 32 rows starting at (x0, y0)
// of C through the warp's staging buffers; `issued` counts the chunks this
// warp has stored so far (buffer = issued % 2).  Lane 0 issues and waits for
// the stores; C edges are clipped by the tensor map.
template <int CH>
__device__ __forceinline__ void acc_tma_store(const CUtensorMap* map_c, uint8_t* warp_stage,
                                              int lane, const uint32_t (&r)[CH][32], int x0,
                                              int y0, int& issued) {
#pragma unroll
  for (int q = 0; q < CH; ++q) {
    uint8_t* buf = warp_stage + (issued & 1) * kEpiChunkBytes;
    if (lane == 0) bulk_wait_group_read<1>();  // the store that used this buffer has read it
    __syncwarp();
    stage_chunk(buf, lane, r[q]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map_c, x0 + 32 * q, y0, buf);
      bulk_commit_group();
    }
    ++issued;
  }
}

// CH x 32 consecutive accumulator columns of this warp's 32 lanes, loaded
// with CH tcgen05.ld and one wait (one round trip).
template <int CH>
__device__ __forceinline__ void acc_load(uint32_t taddr, uint32_t (&r)[CH][32]) {
#pragma unroll
  for (int q = 0; q < CH; ++q) tmem_ld_32cols(taddr + 32 * q, r[q]);
  tmem_wait_ld();
}

// Store CH x 32 loaded columns to row `dst` (column col0 of C) up to column n:
// 16-byte streaming stores where the row allows it, element stores on a
// ragged right edge or unaligned rows.
template <int CH>
__device__ __forceinline__ void acc_store(uint32_t* dst, const uint32_t (&r)[CH][32], int col0,
                                          int n, bool vec) {
#pragma unroll
  for (int q = 0; q < CH; ++q) {
    const int c = col0 + 32 * q;
    if (c >= n) break;
    if (vec && c + 32 <= n) {
#pragma unroll
      for (int v = 0; v < 8; ++v)
        st_stream_u4(dst + 32 * q + 4 * v, r[q][4 * v], r[q][4 * v + 1], r[q][4 * v + 2],
                     r[q][4 * v + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (c + e < n) dst[32 * q + e] = r[q][e];
    }
  }
}

}  // namespace gemm_detail
}  // namespace tcb
