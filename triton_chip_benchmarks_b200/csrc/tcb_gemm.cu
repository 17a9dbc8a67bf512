// Dense GEMM on 5th-generation tensor cores (sm_100a): C = A . B^T.
//
// A [M][K] and B [N][K] are K-contiguous ("TN"); C [M][N] is fp32 (int32 for
// INT8).  MX FP4 operands are E2M1 packed two per byte along K with one E8M0
// scale per 32 elements along K (SA [M][K/32], SB [N][K/32]).  Any M and N, and
// any K whose rows are whole 16-byte units: edge tiles load zeros past the
// matrix (TMA out-of-bounds fill) and store only the rows and columns inside.
//
// Persistent kernel, one CTA per SM, 256 x 256 output tiles (two M=128
// accumulators sharing each B tile; 128 x 256 for MX FP4), warp-specialised:
//   warp 0      TMA producer: per 128-byte K block, A [128 x 128 B] and
//               B [256 x 128 B] tiles (SWIZZLE_128B) into a ring of STAGES
//               shared-memory stages, completing on loaded[stage];
//   warp 1      MMA issuer: waits loaded[stage] (and full[stage] for MX
//               scales), issues the block's four
//               tcgen05.mma (M=128, N=256, K=32 B each) into one tensor-memory
//               accumulator, commits to empty[stage]; after the last block
//               commits to acc_full;
//   warps 2-5   epilogue: wait acc_full, tcgen05.ld their 32 lanes x 256
//               columns, store C, arrive acc_empty;
//   warps 6-9   (MX FP4 only) scale writers: the producer also brings each
//               block's packed E8M0 scales into the stage (bulk copies); the
//               scale warps move them from shared memory into a tensor-memory
//               scale ring slot (same stage index) and arrive on full[stage].
//               (Copying them with tcgen05.cp from the MMA thread instead ran
//               3-15 % slower at M <= 128: the copies take tensor-pipe time.)
// Tiles are visited in groups of 8 row-blocks so concurrent tiles share
// operands in L2; C is written with streaming (evict-first) stores.
// Every wait is bounded; a timeout raises a CTA-wide abort flag so all roles
// leave their loops, and tensor memory is released at the end.
//
// Counterpart in the reference suite: the application GEMM of run_gemm /
// _gemm_kernel (bench_tensor.py:172-209, 1509-1595); the MX FP4 GEMM has no
// counterpart there (FP4 GEMM is refused at bench_tensor.py:1406-1407).
#include <cudaTypedefs.h>

#include "tcb_device.cuh"
#include "tcb_gemm_common.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

using namespace gemm_detail;

}  // namespace

int gemm_pair_run(const void* A, const void* B, const void* SA, const void* SB, void* C, int M,
                  int N, int K, int blocks, int* status, uint32_t idesc, const DeviceFacts& facts,
                  cudaStream_t stream);
int gemm_pair_info(tcb_kernel_info_t* out);

// cuTensorMapEncodeTiled from the driver, resolved once (thread-safe static
// initialisation); null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

namespace {

// Tile geometry: HALVES M=128 accumulators share each B tile.  A 256 x 256
// tile (two halves) feeds the tensor cores with 64 KB per 1024 MMA cycles
// instead of 48 KB per 512 for 128 x 256, i.e. a third less operand traffic
// per FLOP; it fills all 512 tensor-memory columns, so MX FP4 (whose scales
// also live in tensor memory) uses one half.
template <int HALVES, bool SCALED = false>
struct Tile {
  static constexpr int kM = 128 * HALVES;
  static constexpr int kStageA = kM * kBlockBytes;
  static constexpr int kStageB = kTileN * kBlockBytes;
  // MX FP4: the packed E8M0 scales of the block (A: kM x 8 B, B: 256 x 8 B).
  static constexpr int kStageS = SCALED ? (kM + kTileN) * 8 : 0;
  static constexpr int kStageBytes = kStageA + kStageB + kStageS;
  static constexpr int kRing = kSmemBudget - kEpiSmem;  // the rest stages C for TMA stores
  static constexpr int kStages = kRing / kStageBytes > 6 ? 6 : kRing / kStageBytes;
  static constexpr int kSmem = kStages * kStageBytes + kEpiSmem + 1024;
};

template <int KIND>
__device__ __forceinline__ void gemm_mma(uint32_t d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate, uint32_t tsfa,
                                         uint32_t tsfb) {
  if constexpr (KIND == gF16 || KIND == gBF16) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == gTF32) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == gI8) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (KIND == gE4M3) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, "
                 "[%5], [%6], p;\n\t}" ::"r"(d),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  }
}

template <int KIND, int HALVES>
__global__ void __launch_bounds__((6 + kScaleWarps) * 32, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, const GemmArgs args) {
  constexpr bool kScaled = KIND == gMXF4;
  using T = Tile<HALVES, kScaled>;
  constexpr int kStages = T::kStages;
  constexpr int kStageA = T::kStageA;
  constexpr int kStageBytes = T::kStageBytes;
  constexpr int kTileM = T::kM;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t loaded[kMaxStages];  // TMA bytes of the stage landed
  __shared__ __align__(8) uint64_t full[kMaxStages];    // MX scales written to tensor memory
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ __align__(8) uint64_t acc_empty;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = args.tiles_m * args.tiles_n;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_a);
    prefetch_tensormap(&map_b);
    if (args.tma_store) prefetch_tensormap(&map_c);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&loaded[s], 1);
      mbar_init(&full[s], kScaleWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty, kEpilogueWarps);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, args.tiles_m, args.tiles_n, &tm, &tn);
        for (int kb = 0; kb < args.kblocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t phase = static_cast<uint32_t>(it / kStages) & 1u;
          if (!wait_or_abort(&empty[s], phase ^ 1u, &abort_flag, args.status)) break;
          uint8_t* stage = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&loaded[s], kStageBytes);
          tma_load_2d(stage, &map_a, kb * kBlockBytes, tm * kTileM, &loaded[s]);
          tma_load_2d(stage + kStageA, &map_b, kb * kBlockBytes, tn * kTileN, &loaded[s]);
          if constexpr (kScaled) {
            // Packed scales: one contiguous KiB per 128 rows and K block.
            const size_t rb_bytes = static_cast<size_t>(args.kblocks) * 1024;
            uint8_t* ss = stage + kStageA + T::kStageB;
            bulk_load_1d(ss, args.sa + tm * rb_bytes + kb * 1024, 1024, &loaded[s]);
            bulk_load_1d(ss + 1024, args.sb + (2 * tn) * rb_bytes + kb * 1024, 1024, &loaded[s]);
            bulk_load_1d(ss + 2048, args.sb + (2 * tn + 1) * rb_bytes + kb * 1024, 1024,
                         &loaded[s]);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint64_t desc_const = smem_desc(0, 16, 8 * kBlockBytes, 2u);
      const uint32_t smem0 = smem_addr(smem) >> 4;
      int it = 0, ti = 0;
      for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x, ++ti) {
        if (!wait_or_abort(&acc_empty, (static_cast<uint32_t>(ti) & 1u) ^ 1u, &abort_flag,
                           args.status))
          break;
        tc_fence_after();
        for (int kb = 0; kb < args.kblocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t phase = static_cast<uint32_t>(it / kStages) & 1u;
          if (!wait_or_abort(&loaded[s], phase, &abort_flag, args.status)) break;
          if constexpr (kScaled) {
            if (!wait_or_abort(&full[s], phase, &abort_flag, args.status)) break;
          }
          tc_fence_after();
          const uint32_t a_lo = smem0 + static_cast<uint32_t>(s * kStageBytes >> 4);
          const uint32_t b_lo = a_lo + (kStageA >> 4);
          const uint32_t sf = tbase + kAccCols + static_cast<uint32_t>(s * kSfStageCols);
#pragma unroll
          for (int k = 0; k < kStepsPerBlock; ++k) {
            const uint64_t bd = desc_const | (b_lo + static_cast<uint32_t>(k * 2));
#pragma unroll
            for (int h = 0; h < HALVES; ++h) {
              // Half h of A starts 128 rows (16 KB) further into the stage.
              const uint64_t ad =
                  desc_const | (a_lo + static_cast<uint32_t>(h * (128 * kBlockBytes >> 4) + k * 2));
              gemm_mma<KIND>(tbase + h * kAccCols, ad, bd,
                             kScaled ? sf_idesc(args.idesc, k) : args.idesc, (kb | k) != 0,
                             sf_cols_a(sf, k), sf_cols_b(sf, k));
            }
          }
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full);
      }
    }
    __syncwarp();
  } else if (warp < 2 + kEpilogueWarps) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    uint8_t* epi_stage = smem + kStages * kStageBytes + (warp - 2) * kEpiWarpBytes;
    int ti = 0, issued = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++ti) {
      if (!wait_or_abort(&acc_full, static_cast<uint32_t>(ti) & 1u, &abort_flag, args.status))
        break;
      tc_fence_after();
      int tm, tn;
      tile_coords(t, args.tiles_m, args.tiles_n, &tm, &tn);
      // 64-column round trips per M=128 half.  The accumulator is released
      // once its last columns are in registers, so C traffic overlaps the
      // next tile's MMAs.
      uint32_t r[kEpiChunks][32];
#pragma unroll 1
      for (int h = 0; h < HALVES; ++h) {
        const int row0 = tm * kTileM + 128 * h + 32 * quarter;
        const uint32_t taddr = tbase + ((32u * quarter) << 16) + h * kAccCols;
        const int row = row0 + lane;
        const bool row_in = row < args.m;
        uint32_t* dst = args.c + static_cast<size_t>(row) * args.n + tn * kTileN;
#pragma unroll 1
        for (int c0 = 0; c0 < kTileN; c0 += 32 * kEpiChunks) {
          acc_load<kEpiChunks>(taddr + c0, r);
          if (h + 1 == HALVES && c0 + 32 * kEpiChunks == kTileN) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty);
          }
          if (args.tma_store)
            acc_tma_store<kEpiChunks>(&map_c, epi_stage, lane, r, tn * kTileN + c0, row0, issued);
          else if (row_in)
            acc_store<kEpiChunks>(dst + c0, r, tn * kTileN + c0, args.n, args.vec_store);
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();  // C stores complete before the CTA retires
  } else if (kScaled) {
    // ------------------------------------------------------ scale writers
    // The producer brings each block's packed scales into the stage with the
    // operands; lane l takes rows 32j+l (8 bytes each) from shared memory and
    // writes them into the tensor-memory scale ring slot of the same stage.
    const int quarter = warp & 3;
    const uint32_t lane_base = tbase + ((32u * quarter) << 16) + kAccCols;
    int it = 0;
    for (int t = blockIdx.x; t < tiles && !abort_flag; t += gridDim.x) {
      for (int kb = 0; kb < args.kblocks; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t phase = static_cast<uint32_t>(it / kStages) & 1u;
        if (!wait_or_abort(&loaded[s], phase, &abort_flag, args.status)) break;
        const uint8_t* ss = smem + s * kStageBytes + kStageA + T::kStageB + lane * 16;
        write_scale_block(lane_base + static_cast<uint32_t>(s * kSfStageCols), ss, ss + 1024,
                          ss + 2048);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

using GemmFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, GemmArgs);

// MX FP4 uses 128 x 256 tiles (its scales need tensor-memory columns); the
// other kinds use 256 x 256 unless M fits in one 128-row tile.
// 256-row tiles halve the operand traffic per FLOP but also the tile count:
// they are used only when there are at least as many of them as SMs, so a
// 2048 x 2048 problem (64 such tiles) runs as 128 tiles of 128 x 256 instead of
// leaving more than half the SMs idle.
int gemm_halves(int kind, int m, int n, int sm_count) {
  if (kind == gMXF4 || m <= 128) return 1;
  const long long tiles256 = static_cast<long long>((m + 255) / 256) * ((n + kTileN - 1) / kTileN);
  return tiles256 >= sm_count ? 2 : 1;
}

GemmFn gemm_fn(int kind, int halves) {
  if (halves == 2) {
    switch (kind) {
      case gF16: return gemm_kernel<gF16, 2>;
      case gBF16: return gemm_kernel<gBF16, 2>;
      case gTF32: return gemm_kernel<gTF32, 2>;
      case gI8: return gemm_kernel<gI8, 2>;
      case gE4M3: return gemm_kernel<gE4M3, 2>;
    }
    return nullptr;
  }
  switch (kind) {
    case gF16: return gemm_kernel<gF16, 1>;
    case gBF16: return gemm_kernel<gBF16, 1>;
    case gTF32: return gemm_kernel<gTF32, 1>;
    case gI8: return gemm_kernel<gI8, 1>;
    case gE4M3: return gemm_kernel<gE4M3, 1>;
    case gMXF4: return gemm_kernel<gMXF4, 1>;
  }
  return nullptr;
}

int gemm_stages(int kind, int halves) {
  if (kind == gMXF4) return Tile<1, true>::kStages;
  return halves == 2 ? Tile<2>::kStages : Tile<1>::kStages;
}

int gemm_smem(int kind, int halves) {
  if (kind == gMXF4) return Tile<1, true>::kSmem;
  return halves == 2 ? Tile<2>::kSmem : Tile<1>::kSmem;
}

int gemm_kind(int dtype) {
  switch (dtype) {
    case TCB_T_FP16: return gF16;
    case TCB_T_BF16: return gBF16;
    case TCB_T_TF32: return gTF32;
    case TCB_T_INT8: return gI8;
    case TCB_T_FP8E4M3: return gE4M3;
    case TCB_T_MXF4: return gMXF4;
  }
  return -1;
}

int gemm_bits(int kind) {
  switch (kind) {
    case gF16:
    case gBF16: return 16;
    case gTF32: return 32;
    case gI8:
    case gE4M3: return 8;
    case gMXF4: return 4;
  }
  return 0;
}

uint32_t gemm_idesc(int kind, int mma_m = 128) {
  uint32_t d = static_cast<uint32_t>(kTileN >> 3) << 17 | static_cast<uint32_t>(mma_m >> 4) << 24;
  if (kind == gMXF4) return d | 1u << 7 | 1u << 10 | 1u << 23;
  uint32_t c_fmt = 1, ab = 0;
  if (kind == gBF16) ab = 1;
  if (kind == gTF32) ab = 2;
  if (kind == gI8) c_fmt = 2, ab = 1;
  return d | c_fmt << 4 | ab << 7 | ab << 10;
}

int gemm_map(CUtensorMap* map, const void* base, long long rows, long long row_bytes,
             int box_rows) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return TCB_ERR_DEVICE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockBytes), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TCB_OK : TCB_ERR_INVALID_ARGUMENT;
}


// C [M][N] of 32-bit elements, 32 x 32 boxes in the SWIZZLE_128B layout the
// epilogue stages; needs N % 4 == 0 (16-byte row pitch) and a 16-byte base.
int gemm_map_c(CUtensorMap* map, void* base, int rows, int cols) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) return TCB_ERR_DEVICE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TCB_OK : TCB_ERR_INVALID_ARGUMENT;
}

// The arithmetic instruction each kind's kernel writes, in the same wording as
// the resident probe's table (operand and accumulator types spelled out).
const char* gemm_instruction(int kind) {
  switch (kind) {
    case gF16: return "tcgen05.mma.cta_group::1.kind::f16 (f16 x f16 -> f32)";
    case gBF16: return "tcgen05.mma.cta_group::1.kind::f16 (bf16 x bf16 -> f32)";
    case gTF32: return "tcgen05.mma.cta_group::1.kind::tf32 (tf32 x tf32 -> f32)";
    case gI8: return "tcgen05.mma.cta_group::1.kind::i8 (s8 x s8 -> s32)";
    case gE4M3: return "tcgen05.mma.cta_group::1.kind::f8f6f4 (e4m3 x e4m3 -> f32)";
    case gMXF4:
      return "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 (e2m1 x e2m1, ue8m0 -> f32)";
  }
  return "";
}

}  // namespace

int gemm_kernel_info(int dtype, int m, int n, tcb_kernel_info_t* out) {
  if (dtype == TCB_T_FP32 || dtype == TCB_T_FP64) return gemm_cuda_core_info(dtype, out);
  const int kind = gemm_kind(dtype);
  if (kind < 0) return TCB_ERR_UNSUPPORTED;
  if (m <= 0) m = 1 << 16;
  if (n <= 0) n = 1 << 16;
  DeviceFacts facts;
  const int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  if (kind == gMXF4 && m > 128) {
    const int prc = gemm_pair_info(out);
    if (prc != TCB_OK) return prc;
    copy_str(out->instruction, sizeof(out->instruction),
             "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 (e2m1 x e2m1, ue8m0 -> f32)");
    copy_str(out->execution_kind, sizeof(out->execution_kind), "tensor");
    return TCB_OK;
  }
  const int halves = gemm_halves(kind, m, n, facts.sm_count);
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(gemm_fn(kind, halves))) !=
      cudaSuccess)
    return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = gemm_smem(kind, halves);
  out->threads_per_block = (6 + kScaleWarps) * 32;
  out->tensor_core = 1;
  out->pipeline_stages = gemm_stages(kind, halves);
  out->tile_m = 128 * halves;
  out->tile_n = kTileN;
  out->cluster_ctas = 1;
  copy_str(out->instruction, sizeof(out->instruction), gemm_instruction(kind));
  copy_str(out->execution_kind, sizeof(out->execution_kind), "tensor");
  return TCB_OK;
}

// Packed E8M0 layout read by the GEMM: rows padded to a multiple of 256 and
// groups to a multiple of 8 (padding = 127, scale 1.0, so zero-filled operand
// tails stay zero), then one 1 KB block per 128 rows and 8 groups (one 128-byte
// K block of E2M1 codes), made of two 512-byte halves (groups 0-3, 4-7) in
// which lane l = r % 32 owns 16 bytes: the four groups of rows l, 32+l, 64+l,
// 96+l, in that order.
//   dst[((r/128) * (groups_p/8) + g/8) * 1024 + (g%8/4) * 512 + (r%32) * 16
//       + (r%128/32) * 4 + g%4] = src[r][g].
// A scale-writer lane reads its 16 bytes of a half with one load, and they are
// exactly its tensor-memory words for two MMA K steps; a half is also the
// 32-row x 16-byte source format of tcgen05.cp.32x128b.warpx4.  Threads walk
// dst in order, so the stores are coalesced.
__global__ void mx_scales_pack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                      int rows, int groups, long long total, int group_blocks) {
  for (long long o = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; o < total;
       o += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long block = o >> 10;
    const int within = static_cast<int>(o & 1023);
    const long long r = (block / group_blocks) * 128 + ((within >> 2) & 3) * 32 + ((within >> 4) & 31);
    const int g = static_cast<int>(block % group_blocks) * 8 + (within >> 9) * 4 + (within & 3);
    dst[o] = r < rows && g < groups ? src[r * groups + g] : static_cast<uint8_t>(127);
  }
}

long long mx_packed_bytes(int rows, int groups) {
  return ((static_cast<long long>(rows) + 255) / 256 * 256) * ((groups + 7) / 8 * 8);
}

}  // namespace tcb

using namespace tcb;

extern "C" long long tcb_mx_scales_packed_bytes(int rows, int groups) {
  if (rows <= 0 || groups <= 0) return TCB_ERR_INVALID_ARGUMENT;
  return mx_packed_bytes(rows, groups);
}

extern "C" int tcb_mx_scales_pack(const void* src, void* dst, int rows, int groups,
                                  tcb_stream_t stream) {
  if (src == nullptr || dst == nullptr || rows <= 0 || groups <= 0) return TCB_ERR_INVALID_ARGUMENT;
  if (!aligned(dst, 16)) return TCB_ERR_ALIGNMENT;
  const long long total = mx_packed_bytes(rows, groups);
  clear_stale_error();
  mx_scales_pack_kernel<<<512, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), rows, groups, total,
      (groups + 7) / 8);
  return launch_status();
}

extern "C" int tcb_gemm(int dtype, const void* A, const void* B, const void* SA, const void* SB,
                        void* C, int M, int N, int K, int blocks, int* status_dev,
                        tcb_stream_t stream) {
  if (A == nullptr || B == nullptr || C == nullptr || M <= 0 || N <= 0 || K <= 0 || blocks < 0)
    return TCB_ERR_INVALID_ARGUMENT;
  if (dtype == TCB_T_FP32 || dtype == TCB_T_FP64) {
    DeviceFacts facts;
    int rc = current_device_facts(&facts);
    if (rc != TCB_OK) return rc;
    if (facts.major != 10) return TCB_ERR_UNSUPPORTED;
    return gemm_cuda_core(dtype, A, B, C, M, N, K, reinterpret_cast<cudaStream_t>(stream));
  }
  const int kind = gemm_kind(dtype);
  if (kind < 0) return TCB_ERR_UNSUPPORTED;
  // Rows of A and B are TMA rows: their byte length must be a multiple of 16.
  // M, N and the K tail are free (zero-filled loads, masked stores).
  const long long kbits = static_cast<long long>(K) * gemm_bits(kind);
  if (kbits % 128) return TCB_ERR_UNSUPPORTED;
  if (kind == gMXF4 && (SA == nullptr || SB == nullptr)) return TCB_ERR_INVALID_ARGUMENT;
  if (!aligned(A, 16) || !aligned(B, 16) || !aligned(C, 4)) return TCB_ERR_ALIGNMENT;
  if (kind == gMXF4 && (!aligned(SA, 16) || !aligned(SB, 16))) return TCB_ERR_ALIGNMENT;
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  if (facts.major != 10) return TCB_ERR_UNSUPPORTED;
  const long long kbytes = kbits / 8;
  if (kind == gMXF4 && M > 128) {
    // CTA pairs: 256 x 256 tiles, each CTA loading 128 rows of A and of B.
    return gemm_pair_run(A, B, SA, SB, C, M, N, K, blocks, status_dev, gemm_idesc(kind, 256),
                         facts, reinterpret_cast<cudaStream_t>(stream));
  }
  const int halves = gemm_halves(kind, M, N, facts.sm_count);
  const int tile_m = 128 * halves;
  CUtensorMap map_a, map_b;
  if ((rc = gemm_map(&map_a, A, M, kbytes, tile_m)) != TCB_OK) return rc;
  if ((rc = gemm_map(&map_b, B, N, kbytes, kTileN)) != TCB_OK) return rc;
  GemmArgs args;
  args.sa = static_cast<const uint8_t*>(SA);
  args.sb = static_cast<const uint8_t*>(SB);
  args.c = static_cast<uint32_t*>(C);
  args.status = status_dev;
  args.m = M;
  args.n = N;
  args.kbytes = static_cast<int>(kbytes);
  args.kgroups = K / 32;
  args.tiles_m = (M + tile_m - 1) / tile_m;
  args.tiles_n = (N + kTileN - 1) / kTileN;
  args.kblocks = static_cast<int>((kbytes + kBlockBytes - 1) / kBlockBytes);
  args.vec_store = N % 4 == 0 && aligned(C, 16);
  CUtensorMap map_c{};
  args.tma_store = args.vec_store && gemm_map_c(&map_c, C, M, N) == TCB_OK;
  args.idesc = gemm_idesc(kind);
  GemmFn fn = gemm_fn(kind, halves);
  const int smem = gemm_smem(kind, halves);
  static DeviceIntCache cap_cache[6][2];
  const int cap = cap_cache[kind][halves - 1].get(facts.device, [&] {
    return raise_dynamic_smem(reinterpret_cast<const void*>(fn), facts.max_smem_optin);
  });
  if (cap < smem) return TCB_ERR_RESOURCE;
  const int tiles = args.tiles_m * args.tiles_n;
  if (blocks == 0) blocks = facts.sm_count;
  if (blocks > tiles) blocks = tiles;
  clear_stale_error();
  fn<<<blocks, (6 + kScaleWarps) * 32, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      map_a, map_b, map_c, args);
  return launch_status();
}
