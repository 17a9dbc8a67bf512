// Resident-operand matrix probes without a tcgen05 kind (sm_100a):
//   * FP64 on the double-precision MMA path: mma.sync.aligned.m16n8k4 .f64,
//     operands staged once in shared memory in fragment order;
//   * IEEE FP32 and FP64 on the SIMT path: register-blocked fma.rn.f32 /
//     fma.rn.f64 outer products (B200 has no IEEE-FP32 tensor instruction);
//   * IEEE FP32 on the SIMT path with the operands held in registers.
// All keep A and B resident on chip (shared memory, or registers for the
// last) and accumulate C += A . B^T `iterations` times in registers; the CTA
// tile is covered by consecutive register-sized passes, each receiving all
// iterations.
//
// Counterpart in the reference suite: _tensor_peak_kernel
// (bench_tensor.py:406-449) for the fp64 and IEEE-fp32 rows, whose Triton
// lowering is mma.sync f64 and fma.rn.f32 respectively.
#include "tcb_device.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

constexpr int kSimtThreads = 256;
constexpr int kDmmaThreads = 256;

struct SimtArgs {
  const void* a;  // [blocks][M][K]
  const void* b;  // [chains][blocks][N][K]
  void* c;        // [chains][blocks][M][N]
  int blocks, tile_m, tile_n, tile_k, chains, iterations;
};

// ------------------------------------------------------------------ SIMT
// 256 threads as a 16 x 16 grid; each thread owns an 8 x 8 register tile
// made of VEC-wide column groups, so one pass covers 128 x 128 outputs.
// Shared memory holds A^T and B^T in 128-wide pass panels, [pass][K][128],
// so that each thread's eight rows (or columns) for one k are two to four
// 16-byte loads at a compile-time stride (runtime tile extents in the inner
// loop cost address arithmetic and registers: 53.9 vs 58.6 TFLOP/s for FP32).
template <typename T>
__device__ __forceinline__ void fma_rn(T& acc, T a, T b);
template <>
__device__ __forceinline__ void fma_rn<float>(float& acc, float a, float b) {
  asm("fma.rn.f32 %0, %1, %2, %0;" : "+f"(acc) : "f"(a), "f"(b));
}
template <>
__device__ __forceinline__ void fma_rn<double>(double& acc, double a, double b) {
  asm("fma.rn.f64 %0, %1, %2, %0;" : "+d"(acc) : "d"(a), "d"(b));
}

constexpr int kPass = 128;  // rows / columns of one register pass

// FP32 tiles fit two CTAs per SM (128 registers); FP64 tiles need one.
// TM, TN > 0 fix the tile extents at compile time (the pass loops then unroll
// and their addressing leaves the inner loop: 57.6 vs 55.2 TFLOP/s for FP32);
// 0 takes them from the arguments.
template <typename T, int K, int TM = 0, int TN = 0>
__global__ void __launch_bounds__(kSimtThreads, sizeof(T) == 4 ? 2 : 1)
    simt_peak_kernel(const SimtArgs args) {
  constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte shared load
  constexpr int GROUPS = 8 / VEC;      // column groups per thread
  constexpr int kPanel = K * kPass;    // elements of one [K][128] panel
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int M = TM > 0 ? TM : args.tile_m, N = TN > 0 ? TN : args.tile_n;
  const int passes_m = M / kPass, passes_n = N / kPass;
  T* sA = reinterpret_cast<T*>(smem_raw);  // [passes_m][K][128]
  T* sB = sA + passes_m * kPanel;          // [chains][passes_n][K][128]
  const int blk = blockIdx.x;
  const T* gA = static_cast<const T*>(args.a) + static_cast<size_t>(blk) * M * K;
  for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
    const int m = i / K, k = i - m * K;
    sA[(m / kPass) * kPanel + k * kPass + (m % kPass)] = gA[i];
  }
  for (int c = 0; c < args.chains; ++c) {
    const T* gB = static_cast<const T*>(args.b) +
                  static_cast<size_t>(c * args.blocks + blk) * N * K;
    T* sBc = sB + c * passes_n * kPanel;
    for (int i = threadIdx.x; i < N * K; i += blockDim.x) {
      const int n = i / K, k = i - n * K;
      sBc[(n / kPass) * kPanel + k * kPass + (n % kPass)] = gB[i];
    }
  }
  __syncthreads();

  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  for (int c = 0; c < args.chains; ++c) {
    for (int pm = 0; pm < passes_m; ++pm) {
      for (int pn = 0; pn < passes_n; ++pn) {
        const T* a_base = sA + pm * kPanel;
        const T* b_base = sB + (c * passes_n + pn) * kPanel;
        T acc[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = T(0);
#pragma unroll 1
        for (int it = 0; it < args.iterations; ++it) {
          // A modest unroll keeps the shared loads of one k ahead of the
          // FMAs without hoisting all K steps' operands into registers.
#pragma unroll 2
          for (int k = 0; k < K; ++k) {
            T av[8], bv[8];
#pragma unroll
            for (int g = 0; g < GROUPS; ++g) {
              const int off = g * 16 * VEC + VEC * ty;
              const int offb = g * 16 * VEC + VEC * tx;
              if constexpr (VEC == 4) {
                const float4 x = *reinterpret_cast<const float4*>(a_base + k * kPass + off);
                const float4 y = *reinterpret_cast<const float4*>(b_base + k * kPass + offb);
                av[4 * g + 0] = x.x; av[4 * g + 1] = x.y; av[4 * g + 2] = x.z; av[4 * g + 3] = x.w;
                bv[4 * g + 0] = y.x; bv[4 * g + 1] = y.y; bv[4 * g + 2] = y.z; bv[4 * g + 3] = y.w;
              } else {
                const double2 x = *reinterpret_cast<const double2*>(a_base + k * kPass + off);
                const double2 y = *reinterpret_cast<const double2*>(b_base + k * kPass + offb);
                av[2 * g + 0] = x.x; av[2 * g + 1] = x.y;
                bv[2 * g + 0] = y.x; bv[2 * g + 1] = y.y;
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
              for (int j = 0; j < 8; ++j) fma_rn<T>(acc[i][j], av[i], bv[j]);
          }
        }
        // Row (or column) index of register slot i: group i/VEC, lane i%VEC.
        T* gC = static_cast<T*>(args.c) + static_cast<size_t>(c * args.blocks + blk) * M * N;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = pm * kPass + (i / VEC) * 16 * VEC + VEC * ty + (i % VEC);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = pn * kPass + (j / VEC) * 16 * VEC + VEC * tx + (j % VEC);
            gC[static_cast<size_t>(row) * N + col] = acc[i][j];
          }
        }
      }
    }
  }
}

// --------------------------------------------------- SIMT, register-resident
// IEEE FP32 (and FP64) with the operands held in registers for the whole
// reissue loop.  Each lane owns one k of a 16 x 8 output tile (8 x 8 for
// FP64), i.e. 16 A values, 8 B values and 16 x 8 partial sums (152 live
// registers; FP64 8 + 8 + 64 doubles, 160), and the K lanes of a group share
// that tile, so one 256-thread pass covers 32 x (1024 / K) outputs (FP64:
// 32 x (512 / K)).  The loop body is 128 fma.rn.f32 (64 fma.rn.f64) in
// serpentine order (row i left to right, row i + 1 right to left): every FMA
// shares its A or its B register with the one before it, the last FMA of an
// iteration shares B with the first of the next, and an accumulator is reused
// only a whole tile of FMAs later.  After the last iteration the K partial
// sums are added by a butterfly all-reduce (a reduce-scatter, with fewer
// shuffles, changed the loop's register assignment and cost a quarter of the
// rate) and the group's first lane stores the tile.  A and B are staged once
// into shared memory; each pass copies its fragments from there.
constexpr int kRegThreads = 256;
constexpr int kRegPassM = 32;  // pass rows

template <typename T>
struct RegTile {                                        // output tile of one lane group
  static constexpr int kRows = sizeof(T) == 4 ? 16 : 8;
  static constexpr int kCols = 8;
};

template <typename T, int K>
constexpr int reg_pass_n() {
  return kRegThreads / K / (kRegPassM / RegTile<T>::kRows) * RegTile<T>::kCols;
}

// TM, TN > 0 fix the tile extents at compile time (0 takes them from the
// arguments), as for the shared-memory kernel.
template <typename T, int K, int TM = 0, int TN = 0>
__global__ void __launch_bounds__(kRegThreads, 1) simt_reg_peak_kernel(const SimtArgs args) {
  constexpr int kRows = RegTile<T>::kRows, kCols = RegTile<T>::kCols;
  constexpr int kPassN = reg_pass_n<T, K>();
  constexpr int kVec = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int kPitch = K + kVec;      // shared row pitch in elements (16-byte multiple)
  constexpr int kVecs = K / kVec;       // 16-byte vectors per operand row
  constexpr int kVals = kRows * kCols;
  static_assert(K == 8 || K == 16 || K == 32, "one k per lane of a group within a warp");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int M = TM > 0 ? TM : args.tile_m, N = TN > 0 ? TN : args.tile_n;
  T* sA = reinterpret_cast<T*>(smem_raw);  // [M][kPitch]
  T* sB = sA + M * kPitch;                 // [chains][N][kPitch]
  const int blk = blockIdx.x;
  const uint4* gA = reinterpret_cast<const uint4*>(static_cast<const T*>(args.a) +
                                                   static_cast<size_t>(blk) * M * K);
  for (int i = threadIdx.x; i < M * kVecs; i += kRegThreads)
    *reinterpret_cast<uint4*>(sA + (i / kVecs) * kPitch + kVec * (i % kVecs)) = gA[i];
  for (int c = 0; c < args.chains; ++c) {
    const uint4* gB = reinterpret_cast<const uint4*>(
        static_cast<const T*>(args.b) + static_cast<size_t>(c * args.blocks + blk) * N * K);
    T* sBc = sB + c * N * kPitch;
    for (int i = threadIdx.x; i < N * kVecs; i += kRegThreads)
      *reinterpret_cast<uint4*>(sBc + (i / kVecs) * kPitch + kVec * (i % kVecs)) = gB[i];
  }
  __syncthreads();

  const int lk = threadIdx.x % K;    // this lane's k
  const int tile = threadIdx.x / K;  // output tile within the pass
  const int tm = tile % (kRegPassM / kRows), tn = tile / (kRegPassM / kRows);
  for (int c = 0; c < args.chains; ++c) {
    const T* sBc = sB + c * N * kPitch;
    T* gC = static_cast<T*>(args.c) + static_cast<size_t>(c * args.blocks + blk) * M * N;
    for (int pm = 0; pm < M / kRegPassM; ++pm) {
      for (int pn = 0; pn < N / kPassN; ++pn) {
        const int row0 = pm * kRegPassM + tm * kRows, col0 = pn * kPassN + tn * kCols;
        T a[kRows], b[kCols], acc[kVals];
#pragma unroll
        for (int i = 0; i < kRows; ++i) a[i] = sA[(row0 + i) * kPitch + lk];
#pragma unroll
        for (int j = 0; j < kCols; ++j) b[j] = sBc[(col0 + j) * kPitch + lk];
#pragma unroll
        for (int v = 0; v < kVals; ++v) acc[v] = T(0);
#pragma unroll 1
        for (int it = 0; it < args.iterations; ++it) {
#pragma unroll
          for (int i = 0; i < kRows; ++i)
#pragma unroll
            for (int jj = 0; jj < kCols; ++jj) {
              const int j = (i & 1) ? kCols - 1 - jj : jj;
              fma_rn<T>(acc[i * kCols + j], a[i], b[j]);
            }
        }
        // Butterfly all-reduce over the K lanes, then the group's first lane
        // stores the tile.
#pragma unroll
        for (int v = 0; v < kVals; ++v)
#pragma unroll
          for (int s = 1; s < K; s <<= 1) acc[v] += __shfl_xor_sync(0xffffffffu, acc[v], s);
        if (lk == 0) {
#pragma unroll
          for (int v = 0; v < kVals; v += kVec) {
            T* dst = gC + static_cast<size_t>(row0 + v / kCols) * N + col0 + v % kCols;
            if constexpr (sizeof(T) == 4)
              *reinterpret_cast<float4*>(dst) =
                  make_float4(acc[v], acc[v + 1], acc[v + 2], acc[v + 3]);
            else
              *reinterpret_cast<double2*>(dst) = make_double2(acc[v], acc[v + 1]);
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------ DMMA
// 8 warps; warp tile 32 x 64 = 2 (m16) x 8 (n8) mma.sync.m16n8k4 tiles.
// Warps are arranged WM x WN (WN = min(N, 256) / 64), one pass covers
// (32*WM) x (64*WN) outputs.  A and B live in shared memory in fragment order:
//   sA[((mt * KS) + ks) * 32 + lane] = {A[16mt+g][4ks+q], A[16mt+g+8][4ks+q]}
//   sB[((np * KS) + ks) * 32 + lane] = {B[8(2np)+g][4ks+q], B[8(2np+1)+g][4ks+q]}
// with g = lane/4, q = lane%4 (B is stored [N][K], i.e. column-major K x N).
__device__ __forceinline__ void dmma_m16n8k4(double (&c)[4], double a0, double a1, double b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5}, {%6}, "
      "{%0, %1, %2, %3};"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a0), "d"(a1), "d"(b0));
}

template <int K>
__global__ void __launch_bounds__(kDmmaThreads, 1) dmma_peak_kernel(const SimtArgs args) {
  constexpr int KS = K / 4;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int M = args.tile_m, N = args.tile_n;
  double2* sA = reinterpret_cast<double2*>(smem_raw);        // (M/16) * KS * 32
  double2* sB = sA + (M / 16) * KS * 32;                     // chains * (N/16) * KS * 32
  const int blk = blockIdx.x;
  const double* gA = static_cast<const double*>(args.a) + static_cast<size_t>(blk) * M * K;
  for (int i = threadIdx.x; i < (M / 16) * KS * 32; i += blockDim.x) {
    const int lane = i & 31, ks = (i >> 5) % KS, mt = (i >> 5) / KS;
    const int g = lane >> 2, q = lane & 3;
    sA[i] = make_double2(gA[(16 * mt + g) * K + 4 * ks + q], gA[(16 * mt + g + 8) * K + 4 * ks + q]);
  }
  for (int c = 0; c < args.chains; ++c) {
    const double* gB = static_cast<const double*>(args.b) +
                       static_cast<size_t>(c * args.blocks + blk) * N * K;
    double2* sBc = sB + c * (N / 16) * KS * 32;
    for (int i = threadIdx.x; i < (N / 16) * KS * 32; i += blockDim.x) {
      const int lane = i & 31, ks = (i >> 5) % KS, np = (i >> 5) / KS;
      const int g = lane >> 2, q = lane & 3;
      sBc[i] = make_double2(gB[(16 * np + g) * K + 4 * ks + q],
                            gB[(16 * np + 8 + g) * K + 4 * ks + q]);
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn_count = (N < 256 ? N : 256) / 64;
  const int wm_count = 8 / wn_count;
  const int wm = warp / wn_count, wn = warp % wn_count;
  const int pass_m = 32 * wm_count, pass_n = 64 * wn_count;
  const int g = lane >> 2, q = lane & 3;
  for (int c = 0; c < args.chains; ++c) {
    const double2* sBc = sB + c * (N / 16) * KS * 32;
    for (int pm = 0; pm < M / pass_m; ++pm) {
      for (int pn = 0; pn < N / pass_n; ++pn) {
        const int mt0 = (pm * pass_m + 32 * wm) / 16;  // first of this warp's two m16 tiles
        const int np0 = (pn * pass_n + 64 * wn) / 16;  // first of this warp's four n16 pairs
        double acc[2][8][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.0;
#pragma unroll 1
        for (int it = 0; it < args.iterations; ++it) {
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
            double2 af[2], bf[4];
#pragma unroll
            for (int i = 0; i < 2; ++i) af[i] = sA[((mt0 + i) * KS + ks) * 32 + lane];
#pragma unroll
            for (int j = 0; j < 4; ++j) bf[j] = sBc[((np0 + j) * KS + ks) * 32 + lane];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                dmma_m16n8k4(acc[i][2 * j], af[i].x, af[i].y, bf[j].x);
                dmma_m16n8k4(acc[i][2 * j + 1], af[i].x, af[i].y, bf[j].y);
              }
          }
        }
        double* gC = static_cast<double*>(args.c) + static_cast<size_t>(c * args.blocks + blk) * M * N;
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int row = 16 * (mt0 + i) + g;
            const int col = 8 * (2 * np0 + j) + 2 * q;
            gC[static_cast<size_t>(row) * N + col] = acc[i][j][0];
            gC[static_cast<size_t>(row) * N + col + 1] = acc[i][j][1];
            gC[static_cast<size_t>(row + 8) * N + col] = acc[i][j][2];
            gC[static_cast<size_t>(row + 8) * N + col + 1] = acc[i][j][3];
          }
      }
    }
  }
}

using SimtFn = void (*)(SimtArgs);

// Tile-specialised instantiations for the common tiles, runtime extents else.
template <typename T, int K>
SimtFn simt_fn_tile(int m, int n) {
  if (m == 128 && n == 128) return simt_peak_kernel<T, K, 128, 128>;
  if (m == 256 && n == 256) return simt_peak_kernel<T, K, 256, 256>;
  if (m == 128 && n == 256) return simt_peak_kernel<T, K, 128, 256>;
  if (m == 256 && n == 128) return simt_peak_kernel<T, K, 256, 128>;
  return simt_peak_kernel<T, K>;
}

template <typename T, int K>
SimtFn simt_reg_fn_tile(int m, int n) {
  if (m == 64 && n == 64) return simt_reg_peak_kernel<T, K, 64, 64>;
  if (m == 128 && n == 128) return simt_reg_peak_kernel<T, K, 128, 128>;
  if (m == 256 && n == 256) return simt_reg_peak_kernel<T, K, 256, 256>;
  return simt_reg_peak_kernel<T, K>;
}

// (kernel, pass columns) of the register-resident kernel; nullptr for an unsupported K.
template <typename T>
SimtFn simt_reg_fn(int k, int m, int n, int* pass_n) {
  switch (k) {
    case 8: *pass_n = reg_pass_n<T, 8>(); return simt_reg_fn_tile<T, 8>(m, n);
    case 16: *pass_n = reg_pass_n<T, 16>(); return simt_reg_fn_tile<T, 16>(m, n);
    case 32: *pass_n = reg_pass_n<T, 32>(); return simt_reg_fn_tile<T, 32>(m, n);
  }
  return nullptr;
}

template <typename T>
SimtFn simt_fn_k(int k, int m, int n) {
  switch (k) {
    case 8: return simt_fn_tile<T, 8>(m, n);
    case 16: return simt_fn_tile<T, 16>(m, n);
    case 32: return simt_fn_tile<T, 32>(m, n);
    case 64: return simt_fn_tile<T, 64>(m, n);
  }
  return nullptr;
}

SimtFn simt_fn(int dtype, int k, int m, int n) {
  if (dtype == TCB_T_FP32) return simt_fn_k<float>(k, m, n);
  if (dtype == TCB_T_FP64) return simt_fn_k<double>(k, m, n);
  return nullptr;
}

SimtFn dmma_fn(int k) {
  switch (k) {
    case 4: return dmma_peak_kernel<4>;
    case 8: return dmma_peak_kernel<8>;
    case 16: return dmma_peak_kernel<16>;
    case 32: return dmma_peak_kernel<32>;
    case 64: return dmma_peak_kernel<64>;
  }
  return nullptr;
}

struct SimtPlan {
  SimtFn fn = nullptr;
  int threads = 0;
  int smem = 0;
  const char* instruction = "";
  bool tensor = false;
};

int simt_plan(int dtype, int variant, int tile_m, int tile_n, int tile_k, int chains,
              int max_smem, SimtPlan* out) {
  SimtPlan p;
  if (chains < 1 || chains > 2) return TCB_ERR_INVALID_ARGUMENT;
  if (variant == TCB_TV_SIMT_REG) {
    if (dtype != TCB_T_FP32 && dtype != TCB_T_FP64) return TCB_ERR_UNSUPPORTED;
    int pass_n = 0;
    p.fn = dtype == TCB_T_FP32 ? simt_reg_fn<float>(tile_k, tile_m, tile_n, &pass_n)
                               : simt_reg_fn<double>(tile_k, tile_m, tile_n, &pass_n);
    if (p.fn == nullptr) return TCB_ERR_UNSUPPORTED;
    if (tile_m < 1 || tile_n < 1 || tile_m % kRegPassM || tile_n % pass_n || tile_m > 512 ||
        tile_n > 512)
      return TCB_ERR_UNSUPPORTED;
    const int es = dtype == TCB_T_FP32 ? 4 : 8;
    p.threads = kRegThreads;
    p.smem = (tile_m + chains * tile_n) * (tile_k + 16 / es) * es;
    p.instruction = dtype == TCB_T_FP32 ? "fma.rn.f32" : "fma.rn.f64";
    p.tensor = false;
  } else if (variant == TCB_TV_SIMT) {
    if (dtype != TCB_T_FP32 && dtype != TCB_T_FP64) return TCB_ERR_UNSUPPORTED;
    if (tile_m % 128 || tile_n % 128 || tile_m > 512 || tile_n > 512) return TCB_ERR_UNSUPPORTED;
    p.fn = simt_fn(dtype, tile_k, tile_m, tile_n);
    if (p.fn == nullptr) return TCB_ERR_UNSUPPORTED;
    const int es = dtype == TCB_T_FP32 ? 4 : 8;
    p.threads = kSimtThreads;
    p.smem = (tile_m + chains * tile_n) * tile_k * es;
    p.instruction = dtype == TCB_T_FP32 ? "fma.rn.f32" : "fma.rn.f64";
    p.tensor = false;
  } else if (variant == TCB_TV_DMMA) {
    if (dtype != TCB_T_FP64) return TCB_ERR_UNSUPPORTED;
    if (tile_n % 64 || tile_n > 512 || tile_n < 64) return TCB_ERR_UNSUPPORTED;
    const int wn = (tile_n < 256 ? tile_n : 256) / 64;
    const int pass_m = 32 * (8 / wn), pass_n = 64 * wn;
    if (tile_m % pass_m || tile_n % pass_n || tile_m > 512) return TCB_ERR_UNSUPPORTED;
    p.fn = dmma_fn(tile_k);
    if (p.fn == nullptr) return TCB_ERR_UNSUPPORTED;
    p.threads = kDmmaThreads;
    p.smem = (tile_m + chains * tile_n) * tile_k * 8;
    p.instruction = "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64";
    p.tensor = true;
  } else {
    return TCB_ERR_UNSUPPORTED;
  }
  if (p.smem > max_smem) return TCB_ERR_RESOURCE;
  *out = p;
  return TCB_OK;
}

}  // namespace

int tc_tensor_peak(int dtype, const void* A, const void* B, const void* SA, const void* SB,
                   void* C, int blocks, int bps, int tile_m, int tile_n, int tile_k, int chains,
                   int iterations, int* status_dev, cudaStream_t stream);
int tc_kernel_info(int dtype, int tile_m, int tile_n, int tile_k, int chains, int bps,
                   tcb_kernel_info_t* out);

int tensor_kernel_info(int dtype, int variant, int tile_m, int tile_n, int tile_k, int chains,
                       int blocks_per_sm, tcb_kernel_info_t* out) {
  if (variant == TCB_TV_TCGEN05)
    return tc_kernel_info(dtype, tile_m, tile_n, tile_k, chains, blocks_per_sm, out);
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  SimtPlan p;
  rc = simt_plan(dtype, variant, tile_m, tile_n, tile_k, chains, facts.max_smem_optin, &p);
  if (rc != TCB_OK) return rc;
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(p.fn)) != cudaSuccess)
    return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = p.smem;
  out->threads_per_block = p.threads;
  out->tensor_core = p.tensor ? 1 : 0;
  copy_str(out->instruction, sizeof(out->instruction), p.instruction);
  copy_str(out->execution_kind, sizeof(out->execution_kind), p.tensor ? "tensor" : "simt");
  return TCB_OK;
}

}  // namespace tcb

using namespace tcb;

extern "C" int tcb_tensor_peak(int dtype, int variant, const void* A, const void* B,
                               const void* SA, const void* SB, void* C, int blocks,
                               int blocks_per_sm, int tile_m, int tile_n, int tile_k, int chains,
                               int iterations, int* status_dev, tcb_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (variant == TCB_TV_TCGEN05) {
    if (dtype == TCB_T_FP32 || dtype == TCB_T_FP64) return TCB_ERR_UNSUPPORTED;
    return tc_tensor_peak(dtype, A, B, SA, SB, C, blocks, blocks_per_sm, tile_m, tile_n, tile_k,
                          chains, iterations, status_dev, s);
  }
  if (A == nullptr || B == nullptr || C == nullptr || blocks <= 0 || iterations < 1)
    return TCB_ERR_INVALID_ARGUMENT;
  if (!aligned(A, 16) || !aligned(B, 16) || !aligned(C, 16)) return TCB_ERR_ALIGNMENT;
  DeviceFacts facts;
  int rc = current_device_facts(&facts);
  if (rc != TCB_OK) return rc;
  SimtPlan p;
  rc = simt_plan(dtype, variant, tile_m, tile_n, tile_k, chains, facts.max_smem_optin, &p);
  if (rc != TCB_OK) return rc;
  const int cap = raise_dynamic_smem(reinterpret_cast<const void*>(p.fn), facts.max_smem_optin);
  if (cap < 0 || p.smem > cap) return TCB_ERR_RESOURCE;
  clear_stale_error();
  SimtArgs args{A, B, C, blocks, tile_m, tile_n, tile_k, chains, iterations};
  p.fn<<<blocks, p.threads, p.smem, s>>>(args);
  (void)blocks_per_sm;
  (void)SA;
  (void)SB;
  (void)status_dev;
  return launch_status();
}
