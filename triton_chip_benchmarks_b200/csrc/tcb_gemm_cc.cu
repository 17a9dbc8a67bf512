// Dense GEMMs for the formats without a tcgen05 kind (sm_100a): C = A . B^T.
//
//   * IEEE FP32 on the FMA pipe (`fma.rn.f32`): B200 has no IEEE-FP32 tensor
//     instruction.  128 x 128 CTA tile, 256 threads, 8 x 8 register tile per
//     thread; K slabs of 8 are fetched into registers one slab ahead and
//     stored transposed (A^T, B^T) into double-buffered shared memory, so each
//     thread reads its 8 rows / 8 columns of one k with two 16-byte loads.
//   * FP64 on the double-precision MMA path (`mma.sync.m16n8k4.f64`): 128 x
//     128 CTA tile, 8 warps of 32 x 64, K slabs of 32 streamed through a
//     3-stage cp.async ring into padded row-major shared memory (row pitch
//     36 doubles, so the fragment loads of a half-warp hit distinct banks).
//
// A [M][K] and B [N][K] are K-contiguous, C [M][N] row-major (fp32 / fp64).
// Any M, N, K: loads past an edge read zeros, stores are masked (the
// reference's masked tails).  Tiles are visited in groups of 8 row-blocks so
// concurrent CTAs share operands in L2.
//
// Counterpart in the reference suite: run_gemm / _gemm_kernel
// (bench_tensor.py:172-209, 1509-1595) for --dtype fp32 (IEEE input
// precision, its default) and --dtype fp64, whose Triton lowering on NVIDIA is
// fma.rn.f32 and mma.sync f64 respectively.
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

constexpr int kCcTile = 128;
constexpr int kCcThreads = 256;
constexpr int kCcGroupM = 8;

struct CcArgs {
  const void* a;  // [M][K]
  const void* b;  // [N][K]
  void* c;        // [M][N]
  int m, n, k;
  int tiles_m, tiles_n;
  int vec_store;  // C rows 16-byte aligned
};

__device__ __forceinline__ void cc_tile_coords(int t, int tiles_m, int tiles_n, int* tm, int* tn) {
  const int per_group = kCcGroupM * tiles_n;
  const int group = t / per_group;
  const int first = group * kCcGroupM;
  const int rows = min(tiles_m - first, kCcGroupM);
  const int r = t - group * per_group;
  *tm = first + r % rows;
  *tn = r / rows;
}

// ------------------------------------------------------------------- FP32
constexpr int kSgK = 8;
constexpr int kSgPitch = kCcTile + 4;  // floats per k row; +4 keeps the transposed stores conflict-free

__device__ __forceinline__ void ffma(float& acc, float a, float b) {
  asm("fma.rn.f32 %0, %1, %2, %0;" : "+f"(acc) : "f"(a), "f"(b));
}

// VEC: rows are 16-byte aligned (K % 4 == 0), so 4 consecutive k are one load.
template <bool VEC>
__device__ __forceinline__ void sg_fetch(const float* row, bool row_ok, int k0, int K,
                                         float (&r)[4]) {
  if constexpr (VEC) {
    if (row_ok && k0 < K) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(row + k0));
      r[0] = v.x, r[1] = v.y, r[2] = v.z, r[3] = v.w;
    } else {
      r[0] = r[1] = r[2] = r[3] = 0.f;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = row_ok && k0 + i < K ? __ldg(row + k0 + i) : 0.f;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kCcThreads, 2) sgemm_kernel(const CcArgs args) {
  __shared__ __align__(16) float sA[2][kSgK][kSgPitch];
  __shared__ __align__(16) float sB[2][kSgK][kSgPitch];
  int tm, tn;
  cc_tile_coords(blockIdx.x, args.tiles_m, args.tiles_n, &tm, &tn);
  const int K = args.k;
  const int tid = threadIdx.x;
  // Loader: thread t fetches k [4(t%2), +4) of tile row t/2 of A and of B.
  const int lr = tid >> 1, lk = (tid & 1) * 4;
  const int arow = tm * kCcTile + lr, brow = tn * kCcTile + lr;
  const bool a_ok = arow < args.m, b_ok = brow < args.n;
  const float* pa = static_cast<const float*>(args.a) + static_cast<size_t>(a_ok ? arow : 0) * K;
  const float* pb = static_cast<const float*>(args.b) + static_cast<size_t>(b_ok ? brow : 0) * K;
  float ra[4], rb[4];
  const int slabs = (K + kSgK - 1) / kSgK;

  sg_fetch<VEC>(pa, a_ok, lk, K, ra);
  sg_fetch<VEC>(pb, b_ok, lk, K, rb);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sA[0][lk + i][lr] = ra[i];
    sB[0][lk + i][lr] = rb[i];
  }
  __syncthreads();

  // Compute: thread (tx, ty) owns rows {4ty..4ty+3, 64+4ty..} and columns
  // {4tx..4tx+3, 64+4tx..} of the tile.
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

#pragma unroll 1
  for (int s = 0; s < slabs; ++s) {
    const int buf = s & 1;
    const bool more = s + 1 < slabs;
    if (more) {
      sg_fetch<VEC>(pa, a_ok, (s + 1) * kSgK + lk, K, ra);
      sg_fetch<VEC>(pb, b_ok, (s + 1) * kSgK + lk, K, rb);
    }
#pragma unroll
    for (int kk = 0; kk < kSgK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sA[buf][kk][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sA[buf][kk][64 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sB[buf][kk][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sB[buf][kk][64 + 4 * tx]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) ffma(acc[i][j], av[i], bv[j]);
    }
    if (more) {
      // buf ^ 1 was last read in the previous slab, which every thread left
      // at the barrier below.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sA[buf ^ 1][lk + i][lr] = ra[i];
        sB[buf ^ 1][lk + i][lr] = rb[i];
      }
    }
    __syncthreads();
  }

  float* C = static_cast<float*>(args.c);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = tm * kCcTile + (i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4);
    if (row >= args.m) continue;
    float* crow = C + static_cast<size_t>(row) * args.n;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = tn * kCcTile + 64 * h + 4 * tx;
      if (args.vec_store && col + 4 <= args.n) {
        *reinterpret_cast<float4*>(crow + col) =
            make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < args.n) crow[col + j] = acc[i][4 * h + j];
      }
    }
  }
}

// ------------------------------------------------------------------- FP64
constexpr int kDgK = 32;       // K per slab (eight m16n8k4 steps)
constexpr int kDgPitch = 36;   // doubles per shared row (== 4 mod 16: conflict-free fragments)
constexpr int kDgStages = 3;
constexpr int kDgStageDoubles = 2 * kCcTile * kDgPitch;  // A and B rows of one slab
constexpr int kDgSmem = kDgStages * kDgStageDoubles * 8;

__device__ __forceinline__ void dmma(double (&c)[4], double a0, double a1, double b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
      "{%0, %1, %2, %3};"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a0), "d"(a1), "d"(b0));
}

// 8-byte asynchronous copy global -> shared; src_bytes = 0 writes a zero.
__device__ __forceinline__ void cp_async_8(void* smem_dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src), "r"(src_bytes)
               : "memory");
}

// 16-byte form (both addresses 16-byte aligned); src_bytes 0, 8 or 16.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src), "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One slab (k0 .. k0+15) of the A and B tiles into stage buffer `dst`.
// VEC: K even and rows 16-byte aligned -> 16-byte copies (4 per thread per
// matrix), otherwise 8-byte copies (8 per thread per matrix).
template <bool VEC>
__device__ __forceinline__ void dg_load_slab(double* dst, const double* A, const double* B,
                                             int row_a0, int row_b0, int M, int N, int K, int k0,
                                             int tid) {
  constexpr int kPer = VEC ? 2 : 1;                    // doubles per copy
  constexpr int kCopies = kCcTile * kDgK / kPer / kCcThreads;  // per thread per matrix
#pragma unroll
  for (int mat = 0; mat < 2; ++mat) {
    const double* src = mat == 0 ? A : B;
    const int row0 = mat == 0 ? row_a0 : row_b0;
    const int rows = mat == 0 ? M : N;
    double* sdst = dst + mat * kCcTile * kDgPitch;
#pragma unroll
    for (int c = 0; c < kCopies; ++c) {
      const int idx = tid + c * kCcThreads;       // copy index within the slab
      const int r = idx / (kDgK / kPer);
      const int kk = (idx % (kDgK / kPer)) * kPer;
      const int grow = row0 + r, gk = k0 + kk;
      const bool ok = grow < rows && gk < K;
      const double* g = ok ? src + static_cast<size_t>(grow) * K + gk : src;
      if constexpr (VEC) {
        // K is even, so a pair starting inside the row lies entirely inside it.
        cp_async_16(sdst + r * kDgPitch + kk, g, ok ? 16u : 0u);
      } else {
        cp_async_8(sdst + r * kDgPitch + kk, g, ok ? 8u : 0u);
      }
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kCcThreads, 1) dgemm_kernel(const CcArgs args) {
  extern __shared__ __align__(16) double dsm[];
  int tm, tn;
  cc_tile_coords(blockIdx.x, args.tiles_m, args.tiles_n, &tm, &tn);
  const double* A = static_cast<const double*>(args.a);
  const double* B = static_cast<const double*>(args.b);
  const int M = args.m, N = args.n, K = args.k;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row_a0 = tm * kCcTile, row_b0 = tn * kCcTile;
  const int slabs = (K + kDgK - 1) / kDgK;

#pragma unroll
  for (int s = 0; s < kDgStages - 1; ++s) {
    if (s < slabs)
      dg_load_slab<VEC>(dsm + s * kDgStageDoubles, A, B, row_a0, row_b0, M, N, K, s * kDgK, tid);
    cp_async_commit();
  }

  const int wm = warp >> 1, wn = warp & 1;  // 4 x 2 warps, warp tile 32 x 64
  const int g = lane >> 2, q = lane & 3;
  double acc[2][8][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.0;

#pragma unroll 1
  for (int s = 0; s < slabs; ++s) {
    cp_async_wait<kDgStages - 2>();
    __syncthreads();  // slab s landed for all threads; slab s-1's buffer is free
    const int next = s + kDgStages - 1;
    if (next < slabs)
      dg_load_slab<VEC>(dsm + (next % kDgStages) * kDgStageDoubles, A, B, row_a0, row_b0, M, N, K,
                        next * kDgK, tid);
    cp_async_commit();
    const double* sA = dsm + (s % kDgStages) * kDgStageDoubles;
    const double* sB = sA + kCcTile * kDgPitch;
#pragma unroll
    for (int ks = 0; ks < kDgK / 4; ++ks) {
      double a0[2], a1[2], bf[8];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        a0[i] = sA[(32 * wm + 16 * i + g) * kDgPitch + 4 * ks + q];
        a1[i] = sA[(32 * wm + 16 * i + g + 8) * kDgPitch + 4 * ks + q];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) bf[j] = sB[(64 * wn + 8 * j + g) * kDgPitch + 4 * ks + q];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) dmma(acc[i][j], a0[i], a1[i], bf[j]);
    }
  }
  cp_async_wait<0>();

  double* C = static_cast<double*>(args.c);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int row = row_a0 + 32 * wm + 16 * i + g + 8 * half;
      if (row >= M) continue;
      double* crow = C + static_cast<size_t>(row) * N;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = row_b0 + 64 * wn + 8 * j + 2 * q;
        if (args.vec_store && col + 2 <= N) {
          *reinterpret_cast<double2*>(crow + col) =
              make_double2(acc[i][j][2 * half], acc[i][j][2 * half + 1]);
        } else {
          if (col < N) crow[col] = acc[i][j][2 * half];
          if (col + 1 < N) crow[col + 1] = acc[i][j][2 * half + 1];
        }
      }
    }
  }
}

}  // namespace

// FP32 (SIMT) and FP64 (DMMA) GEMM behind tcb_gemm.
int gemm_cuda_core(int dtype, const void* A, const void* B, void* C, int M, int N, int K,
                   cudaStream_t stream) {
  if (dtype != TCB_T_FP32 && dtype != TCB_T_FP64) return TCB_ERR_UNSUPPORTED;
  const int es = dtype == TCB_T_FP32 ? 4 : 8;
  if (!aligned(A, es) || !aligned(B, es) || !aligned(C, es)) return TCB_ERR_ALIGNMENT;
  CcArgs args;
  args.a = A;
  args.b = B;
  args.c = C;
  args.m = M;
  args.n = N;
  args.k = K;
  args.tiles_m = (M + kCcTile - 1) / kCcTile;
  args.tiles_n = (N + kCcTile - 1) / kCcTile;
  const long long tiles = static_cast<long long>(args.tiles_m) * args.tiles_n;
  if (tiles > 0x7FFFFFFFLL) return TCB_ERR_UNSUPPORTED;
  // Rows of A and B start 16-byte aligned when the base is and K * es is a multiple of 16.
  const bool vec_in = aligned(A, 16) && aligned(B, 16) && (static_cast<long long>(K) * es) % 16 == 0;
  args.vec_store = aligned(C, 16) && (static_cast<long long>(N) * es) % 16 == 0;
  clear_stale_error();
  if (dtype == TCB_T_FP32) {
    auto fn = vec_in ? sgemm_kernel<true> : sgemm_kernel<false>;
    fn<<<static_cast<int>(tiles), kCcThreads, 0, stream>>>(args);
    return launch_status();
  }
  auto fn = vec_in ? dgemm_kernel<true> : dgemm_kernel<false>;
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  static DeviceIntCache cap_cache[2];
  const int cap = cap_cache[vec_in ? 1 : 0].get(facts.device, [&] {
    return raise_dynamic_smem(reinterpret_cast<const void*>(fn), facts.max_smem_optin);
  });
  if (cap < kDgSmem) return TCB_ERR_RESOURCE;
  fn<<<static_cast<int>(tiles), kCcThreads, kDgSmem, stream>>>(args);
  return launch_status();
}

int gemm_cuda_core_info(int dtype, tcb_kernel_info_t* out) {
  const void* fn = nullptr;
  if (dtype == TCB_T_FP32) fn = reinterpret_cast<const void*>(sgemm_kernel<true>);
  else if (dtype == TCB_T_FP64) fn = reinterpret_cast<const void*>(dgemm_kernel<true>);
  else return TCB_ERR_UNSUPPORTED;
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, fn) != cudaSuccess) return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = dtype == TCB_T_FP64 ? kDgSmem : 0;
  out->threads_per_block = kCcThreads;
  out->tensor_core = dtype == TCB_T_FP64 ? 1 : 0;
  copy_str(out->instruction, sizeof(out->instruction),
           dtype == TCB_T_FP32 ? "fma.rn.f32" : "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64");
  copy_str(out->execution_kind, sizeof(out->execution_kind),
           dtype == TCB_T_FP32 ? "simt" : "tensor");
  return TCB_OK;
}

}  // namespace tcb
