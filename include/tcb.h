/*
 * tcb.h - C ABI of the B200 (sm_100a) chip-peak probe library, libtcb.so.
 *
 * The library holds the device hot paths of the chip metric suite: the
 * resident-operand tensor multiply-add probe, the vector FMA-chain probe and
 * the device copy/read bandwidth probe.  Each entry point below replaces one
 * Triton launch wrapper of the reference suite (huangyiqun/triton_chip_benchmarks);
 * the replaced function is named beside it as file:line.
 *
 * Conventions for every launch entry point:
 *   - Pointers are device pointers owned by the caller.  The library never
 *     allocates or frees device memory and never synchronizes the device on a
 *     launch path, so a launch can be captured into a CUDA graph.
 *   - `stream` is a cudaStream_t (for PyTorch: torch.cuda.current_stream().cuda_stream).
 *   - The return value is TCB_OK (0) or a negative TCB_ERR_* code.  Argument,
 *     capability and resource problems are detected on the host before any
 *     launch.  Device-side waits are bounded; a wait that runs out writes
 *     TCB_ERR_TIMEOUT into `status_dev` (an int32 device word, may be NULL)
 *     and the kernel returns.
 *   - One host thread per process drives one device (the current device).
 */
#ifndef TCB_H_
#define TCB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *tcb_stream_t; /* identical to cudaStream_t */

/* ---------------------------------------------------------------- status */
#define TCB_OK 0
#define TCB_ERR_INVALID_ARGUMENT (-1) /* bad pointer, size, shape or flag */
#define TCB_ERR_UNSUPPORTED (-2)      /* capability: format/tile not provided on this device */
#define TCB_ERR_RESOURCE (-3)         /* configuration exceeds shared/tensor memory or registers */
#define TCB_ERR_LAUNCH (-4)           /* the CUDA launch itself failed */
#define TCB_ERR_DEVICE (-5)           /* a device query failed */
#define TCB_ERR_TIMEOUT (-6)          /* device-side bounded wait ran out (status word only) */
#define TCB_ERR_ALIGNMENT (-7)        /* pointer or size not aligned as the kernel requires */
#define TCB_ERR_SCRATCH_LIMIT (-8)    /* problem too large for the library's fixed scratch array */

/* Human-readable text for a status code (static storage). */
const char *tcb_strerror(int status);
/* Library version and build target, e.g. "tcb 0.1.0 sm_100a". */
const char *tcb_version(void);

/* ------------------------------------------------------------- device */
typedef struct tcb_device_props {
  char name[256];
  int major, minor;          /* compute capability */
  int sm_count;              /* streaming multiprocessors */
  int max_smem_per_block;    /* opt-in dynamic shared memory per CTA, bytes */
  int max_smem_per_sm;       /* shared memory per SM, bytes */
  int regs_per_sm;           /* 32-bit registers per SM */
  int clock_khz;             /* max SM clock */
  int mem_clock_khz;         /* max memory clock */
  int mem_bus_width;         /* bits */
  long long l2_cache_bytes;  /* L2 capacity */
  long long total_mem_bytes; /* device memory capacity */
  long long free_mem_bytes;  /* currently free device memory */
  int driver_version, runtime_version;
} tcb_device_props;

/* Properties of `device`.  Replaces the property probing of setup_device
 * (common.py:214-292) and the capacity probe of probe_device
 * (bench_suite.py:106-114). */
int tcb_device_query(int device, tcb_device_props *out);

/* --------------------------------------------------------- copy / read */
#define TCB_COPY_LDG128 0 /* 128-bit loads/stores, one CTA per piece (or grid-stride) */
#define TCB_COPY_BULK 1   /* bulk-copy engine: global -> shared -> global, one lane per CTA */

/* dst[0:bytes) = src[0:bytes).  Any byte count and alignment is accepted;
 * both kernels need 16-byte aligned pointers and otherwise fall back to a byte
 * loop.  blocks = 0 selects the tuned grid for the variant.  For LDG128,
 * `threads` is the CTA size (0: 768) and each CTA copies a piece of
 * threads x 32 bytes; blocks = 0 launches one CTA per piece, a smaller
 * positive `blocks` walks the pieces grid-stride.  For BULK the CTA is one warp and
 * `threads` is the depth of the shared-memory ring in 32 KiB chunks (2..8,
 * 0: 2; the default grid is 2 CTAs per SM). src and dst must not overlap.
 * A bulk-copy ring wait that runs out writes TCB_ERR_TIMEOUT into
 * `status_dev` (may be NULL; the LDG128 and byte kernels never wait).
 * Replaces launch_copy (bench_bandwidth.py:43-47) and copy_kernel
 * (bench_bandwidth.py:36-40). */
int tcb_copy(const void *src, void *dst, size_t bytes, int variant, int blocks, int threads,
             int *status_dev, tcb_stream_t stream);

#define TCB_READ_FP32 0
#define TCB_READ_FP16 1
#define TCB_READ_BF16 2
/* sink[i] = FP32 sum of src[i*block_elems : (i+1)*block_elems) (the last
 * block may be partial).  block_elems is a power of two in [256, 65536].
 * Replaces launch_read (bench_bandwidth.py:62-67) and read_kernel
 * (bench_bandwidth.py:50-59). */
int tcb_read(const void *src, int dtype, long long elements, float *sink, int block_elems,
             int threads, tcb_stream_t stream);

/* ------------------------------------------------------ vector chains */
#define TCB_V_BF16 0       /* fma.rn.bf16x2, packed pairs */
#define TCB_V_FP16 1       /* fma.rn.f16x2, packed pairs */
#define TCB_V_FP32 2       /* fma.rn.f32 */
#define TCB_V_FP64 3       /* fma.rn.f64 */
#define TCB_V_INT8_DP4A 4  /* dp4a.s32.s32 on int32 words, 8 ops per update */
#define TCB_V_INT32_IMAD 5 /* mad.lo.s32 (int32 wrap), 2 ops per update */
#define TCB_V_INT8_MULADD 6 /* int8 state, (x*a + b) mod 256, 2 ops per update */

/* Eight independent chains per element: out[c][e] = f^iterations(in[c][e])
 * with f(x) = x*coeff[0] + coeff[1+c] (dp4a: f(x) = dot4(x, coeff[0]) + coeff[1+c]).
 * in/out are [8][elements] in the dtype's storage (int32 words for DP4A and
 * IMAD, int8 for MULADD), coeff holds 9 values of the same storage type.
 * elements must equal blocks * threads * elems_per_thread; elems_per_thread
 * is one of 1,2,4,8,16 (even for the packed 16-bit types); unroll is one of
 * 1,2,4,8,16 (any iteration count is accepted).  Replaces launch_vector
 * (bench_vector.py:1032-1051) and vector_fma_kernel (bench_vector.py:182-319). */
int tcb_vector_chains(int dtype, const void *in, void *out, const void *coeff,
                      long long elements, int iterations, int blocks, int threads,
                      int elems_per_thread, int unroll, tcb_stream_t stream);

/* The same chains with the 9 coefficients read from HOST memory during the
 * call (same storage type and order as `coeff` above) and passed to the kernel
 * by value, where the FMAs can take them as constant-bank operands.  Measured
 * on B200: FP32 and FP64 chains are faster this way (FP64 37.0 vs 34.1 TFLOP/s
 * with register-resident coefficients), packed bf16x2/f16x2 and DP4A chains
 * slower (bf16x2 73.4-74.0 vs 74.1-74.3 TFLOP/s; DP4A 148.2 vs 148.5 TOP/s),
 * so callers pick the entry point per dtype.  The reference-side binding
 * copies its device coefficient tensor to the host once, outside timing. */
int tcb_vector_chains_imm(int dtype, const void *in, void *out, const void *coeff_host,
                          long long elements, int iterations, int blocks, int threads,
                          int elems_per_thread, int unroll, tcb_stream_t stream);

/* ------------------------------------------------------ tensor probe */
#define TCB_T_BF16 0
#define TCB_T_FP16 1
#define TCB_T_TF32 2      /* fp32 storage, tcgen05 kind::tf32 */
#define TCB_T_FP32 3      /* IEEE fp32, SIMT FFMA (no IEEE-fp32 tensor instruction exists) */
#define TCB_T_FP64 4
#define TCB_T_INT8 5      /* int8 in, int32 accumulate */
#define TCB_T_FP8E4M3 6   /* e4m3fn in, fp32 accumulate */
#define TCB_T_MXF4 7      /* OCP MX E2M1 packed two per byte (low nibble = even k), E8M0 scales */

#define TCB_TV_TCGEN05 0  /* tcgen05.mma, accumulators in tensor memory */
#define TCB_TV_DMMA 1     /* mma.sync f64 (fp64 only) */
#define TCB_TV_SIMT 2     /* scalar FFMA / DFMA (fp32, fp64), operands read from shared memory */
#define TCB_TV_SIMT_REG 3 /* scalar FFMA / DFMA (fp32, fp64), operands held in registers;
                           * tile_k 8, 16 or 32, tile_m a multiple of 32, tile_n a
                           * multiple of 1024 / tile_k (fp32) or 512 / tile_k (fp64) */

/* Resident-operand probe.  CTA b loads A_b and B_{c,b} (c < chains) once and
 * then accumulates C_{c,b} += A_b . B_{c,b}^T `iterations` times.
 *   A  : [blocks][tile_m][tile_k]            row-major (K contiguous)
 *   B  : [chains][blocks][tile_n][tile_k]    K contiguous (i.e. B^T of the [K][N] operand)
 *   C  : [chains][blocks][tile_m][tile_n]    fp32 (int32 for INT8, fp64 for FP64)
 *   For MXF4 the K axis is packed (tile_k/2 bytes per row) and
 *   SA : [blocks][tile_m][tile_k/32], SB : [blocks][tile_n][tile_k/32] E8M0 bytes.
 * blocks_per_sm is the intended residency (it sizes the tensor-memory share
 * and shared-memory reservation of each CTA).  Replaces _launch_peak
 * (bench_tensor.py:581-600) with _tensor_peak_kernel (bench_tensor.py:406-449)
 * and _tensor_peak_scaled_kernel (bench_tensor.py:452-488). */
int tcb_tensor_peak(int dtype, int variant, const void *A, const void *B, const void *SA,
                    const void *SB, void *C, int blocks, int blocks_per_sm, int tile_m,
                    int tile_n, int tile_k, int chains, int iterations, int *status_dev,
                    tcb_stream_t stream);

/* ------------------------------------------------------------- GEMM */
/* C[M][N] = A[M][K] . B[N][K]^T with A and B K-contiguous, C row-major fp32
 * (int32 for TCB_T_INT8, fp64 for TCB_T_FP64).  dtype: TCB_T_BF16, FP16,
 * TF32, INT8, FP8E4M3, MXF4 on tcgen05; TCB_T_FP32 (IEEE, fma.rn.f32 on the
 * FMA pipe) and TCB_T_FP64 (mma.sync f64) on CUDA cores, which take any M,
 * N, K, element-aligned pointers, and ignore `blocks` and `status_dev`.
 * For MXF4, A and B hold E2M1 codes packed two per byte along K (low nibble =
 * even k) and SA, SB hold the E8M0 scales of A [M][K/32] and B [N][K/32] in
 * the packed layout written by tcb_mx_scales_pack (16-byte aligned).
 * tcgen05 kinds: any M, N >= 1 (edge tiles are masked, like the reference's
 * masked tails); K x element bits must be a multiple of 128 (each row of A and B a whole
 * number of 16-byte units: K % 8 for 16-bit types, % 4 for TF32, % 16 for
 * 8-bit, % 32 for MXF4), otherwise TCB_ERR_UNSUPPORTED.  A, B 16-byte
 * aligned, C 4-byte aligned.  blocks = 0 selects one persistent CTA per SM.
 * Replaces run_gemm / _launch / _gemm_kernel (bench_tensor.py:172-209,
 * 235-246, 1509-1595); the MX FP4 GEMM has no counterpart in the reference
 * (which refuses FP4 GEMM, bench_tensor.py:1406-1407). */
int tcb_gemm(int dtype, const void *A, const void *B, const void *SA, const void *SB, void *C,
             int M, int N, int K, int blocks, int *status_dev, tcb_stream_t stream);

/* Bytes of the packed scale layout for E8M0 scales [rows][groups]:
 * rows rounded up to a multiple of 256 times groups rounded up to a multiple
 * of 8.  Returns TCB_ERR_INVALID_ARGUMENT for non-positive sizes. */
long long tcb_mx_scales_packed_bytes(int rows, int groups);

/* Rearrange E8M0 scales src [rows][groups] (row-major, one byte per 32 K
 * elements) into the layout tcb_gemm reads: rows padded to a multiple of 256
 * and groups to a multiple of 8 with the unit scale 127, then one 1 KB block
 * per 128 rows and 8 groups, in two 512-byte halves (groups 0-3 and 4-7) of
 * 32 x 16 bytes, lane l = r % 32 holding the four groups of rows l, 32+l,
 * 64+l, 96+l:
 * dst[((r/128)*(groups_p/8) + g/8)*1024 + (g%8/4)*512 + (r%32)*16
 *     + (r%128/32)*4 + g%4] = src[r*groups + g].
 * Each half is the shared-memory source of one tensor-memory copy
 * (tcgen05.cp.32x128b.warpx4).  dst holds tcb_mx_scales_packed_bytes(rows,
 * groups) bytes, 16-byte aligned.  Run once per scale tensor (data
 * preparation, not part of the GEMM).  No counterpart in the reference. */
int tcb_mx_scales_pack(const void *src, void *dst, int rows, int groups, tcb_stream_t stream);

/* MX FP4 GEMM that allocates nothing, for callers that cannot allocate device
 * memory (a plugin whose host framework owns all device memory through its
 * own pool, or a path where cudaMalloc/cudaFree and their synchronisation are
 * not allowed).  No counterpart in the reference.
 * Same contract as tcb_gemm(TCB_T_MXF4, ...) except that SA [M][K/32] and
 * SB [N][K/32] are plain row-major E8M0 scales (any alignment): the call packs
 * them into a fixed 8 MiB scratch array in the library's device image, then
 * runs the GEMM, all in order on `stream`.  Limits: K % 32 == 0
 * (TCB_ERR_UNSUPPORTED otherwise), and the packed scales of A and of B, each
 * rounded up to 256 bytes, must fit in 8 MiB (M = N = 16384 at K = 8192 does),
 * otherwise TCB_ERR_SCRATCH_LIMIT before anything is launched.
 * The scratch array is held by every device that loads the library until the
 * process exits.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current); make that first
 * call before any stream capture.  Every call shares the one array and
 * rewrites all of the part it reads: calls whose work overlaps on the GPU
 * (different streams, or other host threads) race on it and must be
 * serialised by the caller. */
int tcb_gemm_mxf4_noalloc(const void *A, const void *B, const void *SA, const void *SB, void *C,
                          int M, int N, int K, int blocks, int *status_dev, tcb_stream_t stream);

/* --------------------------------------------------------- self-test */
/* Runs the library's bounded device-side wait against an mbarrier whose phase
 * can never complete (armed for bytes no copy delivers), with a limit of
 * `limit_ns` (0..1e9).  The kernel must give up, write TCB_ERR_TIMEOUT into
 * `status_dev` (required) and return, leaving the context usable: this is the
 * path every probe kernel takes when one of its waits runs out.  No
 * counterpart in the reference (its Triton kernels have no device waits). */
int tcb_selftest_bounded_wait(long long limit_ns, int *status_dev, tcb_stream_t stream);

/* ------------------------------------------------------- kernel info */
#define TCB_FAMILY_COPY 0
#define TCB_FAMILY_READ 1
#define TCB_FAMILY_VECTOR 2
#define TCB_FAMILY_TENSOR 3
#define TCB_FAMILY_GEMM_FP4 4

typedef struct tcb_kernel_info_t {
  int registers_per_thread;  /* cudaFuncAttributes.numRegs */
  int local_bytes_per_thread; /* cudaFuncAttributes.localSizeBytes (spill indicator) */
  int static_smem_bytes;
  int dynamic_smem_bytes;    /* what the launch requests */
  int max_threads_per_block;
  int threads_per_block;     /* what the launch uses */
  int tensor_core;           /* 1: the arithmetic runs on tensor cores */
  char instruction[128];     /* the arithmetic instruction written in the kernel source */
  char execution_kind[16];   /* "tensor" or "simt" */
  int pipeline_stages;       /* GEMM: shared-memory operand stages of the ring (else 0) */
  int tile_m, tile_n;        /* GEMM: output tile of one CTA or CTA cluster (else 0) */
  int cluster_ctas;          /* GEMM: CTAs that share one output tile (1, or 2 for pairs) */
} tcb_kernel_info_t;

/* Static facts about the kernel a launch with these arguments would run.
 * `a0..a5` are the family's launch parameters:
 *   COPY   : variant, threads
 *   READ   : dtype, threads
 *   VECTOR : dtype, threads, elems_per_thread, unroll, coefficients (0: passed by
 *            value, tcb_vector_chains_imm; 1: from device memory into registers,
 *            tcb_vector_chains)
 *   TENSOR : dtype, variant, tile_m, tile_n, tile_k, chains (blocks_per_sm via a6)
 *   GEMM_FP4 (any GEMM dtype): dtype, M, N (M, N = 0: a large problem); the
 *            kernel tcb_gemm would run for that shape on the current device
 * Replaces the CompiledKernel metadata read by _compiled_info
 * (bench_tensor.py:984-1146) and inspect_assembly (bench_vector.py:623-799). */
int tcb_kernel_info(int family, int a0, int a1, int a2, int a3, int a4, int a5, int a6,
                    tcb_kernel_info_t *out);

#ifdef __cplusplus
}
#endif

#endif /* TCB_H_ */
