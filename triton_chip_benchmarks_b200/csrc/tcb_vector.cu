// Vector FMA-chain probe (sm_100a).
//
// Every element carries CHAINS = 8 independent accumulators that each run the
// recurrence x <- x*a + b_c for `iterations` steps, entirely in registers.
// The update is one hand-written PTX instruction per accumulator and dtype:
//   bf16/fp16  fma.rn.bf16x2 / fma.rn.f16x2 on packed element pairs
//   fp32/fp64  fma.rn.f32 / fma.rn.f64
//   int8 dp4a  dp4a.s32.s32 on int32 words (four int8 products + int32 bias)
//   int32      mad.lo.s32 (int32 wrap-around)
//   int8 mod   mad.lo.s32 followed by a sign-extension of the low byte
// Each thread owns ELEMS elements (ELEMS/2 packed pairs for 16-bit types),
// strided by the block size so every load and store is coalesced.
//
// Counterpart in the reference suite: vector_fma_kernel and its update
// helpers (bench_vector.py:87-319), launched by launch_vector
// (bench_vector.py:1032-1051).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "tcb_device.cuh"
#include "tcb_host.h"
#include "tcb_registry.h"

namespace tcb {
namespace {

constexpr int kChains = 8;

// One accumulator update per dtype.  `Word` is the register type holding one
// accumulator (a packed pair for the 16-bit types).
struct OpBF16 {
  using Word = uint32_t;
  static constexpr int kPack = 2;
  static constexpr int kStorageBytes = 2;
  static constexpr const char* kInstruction = "fma.rn.bf16x2";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("fma.rn.bf16x2 %0, %0, %1, %2;" : "+r"(x) : "r"(a), "r"(b));
  }
};

struct OpFP16 {
  using Word = uint32_t;
  static constexpr int kPack = 2;
  static constexpr int kStorageBytes = 2;
  static constexpr const char* kInstruction = "fma.rn.f16x2";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(x) : "r"(a), "r"(b));
  }
};

struct OpFP32 {
  using Word = float;
  static constexpr int kPack = 1;
  static constexpr int kStorageBytes = 4;
  static constexpr const char* kInstruction = "fma.rn.f32";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("fma.rn.f32 %0, %0, %1, %2;" : "+f"(x) : "f"(a), "f"(b));
  }
};

struct OpFP64 {
  using Word = double;
  static constexpr int kPack = 1;
  static constexpr int kStorageBytes = 8;
  static constexpr const char* kInstruction = "fma.rn.f64";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("fma.rn.f64 %0, %0, %1, %2;" : "+d"(x) : "d"(a), "d"(b));
  }
};

struct OpDP4A {
  using Word = int32_t;
  static constexpr int kPack = 1;
  static constexpr int kStorageBytes = 4;
  static constexpr const char* kInstruction = "dp4a.s32.s32";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("dp4a.s32.s32 %0, %0, %1, %2;" : "+r"(x) : "r"(a), "r"(b));
  }
};

struct OpIMAD {
  using Word = int32_t;
  static constexpr int kPack = 1;
  static constexpr int kStorageBytes = 4;
  static constexpr const char* kInstruction = "mad.lo.s32";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("mad.lo.s32 %0, %0, %1, %2;" : "+r"(x) : "r"(a), "r"(b));
  }
};

// INT8 state held sign-extended in a 32-bit register: (x*a + b) mod 256.
struct OpI8MulAdd {
  using Word = int32_t;
  static constexpr int kPack = 1;
  static constexpr int kStorageBytes = 1;
  static constexpr const char* kInstruction = "mad.lo.s32 + cvt.s32.s8";
  __device__ __forceinline__ static void step(Word& x, Word a, Word b) {
    asm("{\n\t.reg .s32 t;\n\t"
        "mad.lo.s32 t, %0, %1, %2;\n\t"
        "cvt.s32.s8 %0, t;\n\t}"
        : "+r"(x)
        : "r"(a), "r"(b));
  }
};

// Load/store of one accumulator word from storage.
template <typename Op>
struct Mem {
  using Word = typename Op::Word;
  __device__ __forceinline__ static Word load(const void* base, long long idx) {
    return static_cast<const Word*>(base)[idx];
  }
  __device__ __forceinline__ static void store(void* base, long long idx, Word v) {
    static_cast<Word*>(base)[idx] = v;
  }
  // Coefficients as the kernel uses them: packed pairs repeat the scalar.
  __device__ __forceinline__ static Word coeff(const void* c, int i) {
    return static_cast<const Word*>(c)[i];
  }
};

template <>
struct Mem<OpBF16> {
  __device__ __forceinline__ static uint32_t load(const void* base, long long idx) {
    return static_cast<const uint32_t*>(base)[idx];
  }
  __device__ __forceinline__ static void store(void* base, long long idx, uint32_t v) {
    static_cast<uint32_t*>(base)[idx] = v;
  }
  __device__ __forceinline__ static uint32_t coeff(const void* c, int i) {
    const uint32_t h = static_cast<const unsigned short*>(c)[i];
    return h | (h << 16);
  }
};

template <>
struct Mem<OpFP16> : Mem<OpBF16> {};

template <>
struct Mem<OpI8MulAdd> {
  __device__ __forceinline__ static int32_t load(const void* base, long long idx) {
    return static_cast<const int8_t*>(base)[idx];
  }
  __device__ __forceinline__ static void store(void* base, long long idx, int32_t v) {
    static_cast<int8_t*>(base)[idx] = static_cast<int8_t>(v);
  }
  __device__ __forceinline__ static int32_t coeff(const void* c, int i) {
    return static_cast<const int8_t*>(c)[i];
  }
};

// Coefficients {a, b_0..b_7} passed by value: they live in the kernel
// parameter (constant) bank, so the compiler can feed them to the FMA as
// constant-bank operands instead of registers.  For FP64 this matters: a
// DFMA with three register-resident 64-bit operands ran at 92 % of the FP64
// pipe, one with constant-bank coefficients at 99.7 %.
template <typename Op>
struct CoeffImm {
  typename Op::Word v[1 + kChains];
};

// in/out: [8][elements] storage; words are kPack elements wide.  IMM selects
// the coefficient source: the by-value parameter `imm`, or device memory at
// `coeff` (loaded once into registers).
template <typename Op, int ELEMS, int UNROLL, bool IMM>
__global__ void __launch_bounds__(1024)
    chains_kernel(const void* __restrict__ in, void* __restrict__ out,
                  const void* __restrict__ coeff, const __grid_constant__ CoeffImm<Op> imm,
                  long long words_per_chain, int iterations) {
  using Word = typename Op::Word;
  constexpr int kSlots = ELEMS / Op::kPack;
  const long long block_words = static_cast<long long>(blockDim.x) * kSlots;
  const long long first = static_cast<long long>(blockIdx.x) * block_words + threadIdx.x;

  Word x[kChains][kSlots];
#pragma unroll
  for (int c = 0; c < kChains; ++c)
#pragma unroll
    for (int i = 0; i < kSlots; ++i)
      x[c][i] = Mem<Op>::load(in, c * words_per_chain + first + i * blockDim.x);

  Word a_reg{}, b_reg[kChains]{};
  if constexpr (!IMM) {
    a_reg = Mem<Op>::coeff(coeff, 0);
#pragma unroll
    for (int c = 0; c < kChains; ++c) b_reg[c] = Mem<Op>::coeff(coeff, 1 + c);
  }
  // One update of every accumulator.
  auto sweep = [&]() {
#pragma unroll
    for (int c = 0; c < kChains; ++c)
#pragma unroll
      for (int i = 0; i < kSlots; ++i) {
        if constexpr (IMM)
          Op::step(x[c][i], imm.v[0], imm.v[1 + c]);
        else
          Op::step(x[c][i], a_reg, b_reg[c]);
      }
  };

  const int full = iterations / UNROLL;
  const int rest = iterations - full * UNROLL;
#pragma unroll 1
  for (int it = 0; it < full; ++it) {
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) sweep();
  }
#pragma unroll 1
  for (int it = 0; it < rest; ++it) sweep();

#pragma unroll
  for (int c = 0; c < kChains; ++c)
#pragma unroll
    for (int i = 0; i < kSlots; ++i)
      Mem<Op>::store(out, c * words_per_chain + first + i * blockDim.x, x[c][i]);
}

template <typename Op>
using ChainFnT = void (*)(const void*, void*, const void*, CoeffImm<Op>, long long, int);

constexpr int kElemChoices[] = {1, 2, 4, 8, 16};
constexpr int kUnrollChoices[] = {1, 2, 4, 8, 16};

int elem_index(int e) {
  for (int i = 0; i < 5; ++i)
    if (kElemChoices[i] == e) return i;
  return -1;
}
int unroll_index(int u) {
  for (int i = 0; i < 5; ++i)
    if (kUnrollChoices[i] == u) return i;
  return -1;
}

// Table [elems][unroll] of kernel instantiations for one op.  16-bit ops
// have no ELEMS=1 variant (a packed pair holds two elements).
template <typename Op, int E, bool IMM>
struct Row {
  static constexpr ChainFnT<Op> fns[5] = {
      chains_kernel<Op, E, 1, IMM>, chains_kernel<Op, E, 2, IMM>, chains_kernel<Op, E, 4, IMM>,
      chains_kernel<Op, E, 8, IMM>, chains_kernel<Op, E, 16, IMM>};
};

template <typename Op, bool IMM>
ChainFnT<Op> pick(int e, int u) {
  const int ei = elem_index(e), ui = unroll_index(u);
  if (ei < 0 || ui < 0) return nullptr;
  if (Op::kPack == 2 && e == 1) return nullptr;
  switch (e) {
    case 1:
      if constexpr (Op::kPack == 1) return Row<Op, 1, IMM>::fns[ui];
      return nullptr;
    case 2:
      return Row<Op, 2, IMM>::fns[ui];
    case 4:
      return Row<Op, 4, IMM>::fns[ui];
    case 8:
      return Row<Op, 8, IMM>::fns[ui];
    case 16:
      return Row<Op, 16, IMM>::fns[ui];
  }
  return nullptr;
}

// Coefficients as the kernels use them, from host memory in the storage type
// (packed 16-bit pairs repeat the scalar; int8 is sign-extended).
template <typename Op>
CoeffImm<Op> host_coeffs(const void* host) {
  CoeffImm<Op> c{};
  for (int i = 0; i < 1 + kChains; ++i) {
    if constexpr (Op::kPack == 2) {
      const uint32_t h = static_cast<const unsigned short*>(host)[i];
      c.v[i] = h | (h << 16);
    } else if constexpr (Op::kStorageBytes == 1) {
      c.v[i] = static_cast<const int8_t*>(host)[i];
    } else {
      c.v[i] = static_cast<const typename Op::Word*>(host)[i];
    }
  }
  return c;
}

// Launch one op's kernel: `imm_host` (host coefficients, by-value path) or
// `coeff` (device coefficients).
template <typename Op>
int launch_op(int e, int u, const void* in, void* out, const void* coeff, const void* imm_host,
              long long words, int iterations, int blocks, int threads, cudaStream_t s,
              bool query_only, const void** fn_out) {
  // A query asks for the by-value variant with a non-null imm_host and for
  // the register variant with a non-null coeff (neither is dereferenced).
  ChainFnT<Op> fn = imm_host != nullptr ? pick<Op, true>(e, u) : pick<Op, false>(e, u);
  if (fn == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  if (fn_out != nullptr) *fn_out = reinterpret_cast<const void*>(fn);
  if (query_only) return TCB_OK;
  const CoeffImm<Op> imm = imm_host != nullptr ? host_coeffs<Op>(imm_host) : CoeffImm<Op>{};
  clear_stale_error();
  fn<<<blocks, threads, 0, s>>>(in, out, coeff, imm, words, iterations);
  return launch_status();
}

struct OpFacts {
  int pack = 1;
  int storage_bytes = 4;
  const char* instruction = "";
};

// Dispatch on dtype: dtype facts, and (unless `facts_only`) the launch.
int dispatch(int dtype, int e, int u, const void* in, void* out, const void* coeff,
             const void* imm_host, long long words, int iterations, int blocks, int threads,
             cudaStream_t s, bool query_only, const void** fn_out, OpFacts* facts,
             bool facts_only) {
#define TCB_VECTOR_CASE(CODE, OP)                                                           \
  case CODE:                                                                                \
    *facts = {OP::kPack, OP::kStorageBytes, OP::kInstruction};                              \
    if (facts_only) return TCB_OK;                                                          \
    return launch_op<OP>(e, u, in, out, coeff, imm_host, words, iterations, blocks, threads, \
                         s, query_only, fn_out);
  switch (dtype) {
    TCB_VECTOR_CASE(TCB_V_BF16, OpBF16)
    TCB_VECTOR_CASE(TCB_V_FP16, OpFP16)
    TCB_VECTOR_CASE(TCB_V_FP32, OpFP32)
    TCB_VECTOR_CASE(TCB_V_FP64, OpFP64)
    TCB_VECTOR_CASE(TCB_V_INT8_DP4A, OpDP4A)
    TCB_VECTOR_CASE(TCB_V_INT32_IMAD, OpIMAD)
    TCB_VECTOR_CASE(TCB_V_INT8_MULADD, OpI8MulAdd)
    default:
      return TCB_ERR_INVALID_ARGUMENT;
  }
#undef TCB_VECTOR_CASE
}

}  // namespace

int vector_kernel_info(int dtype, int threads, int elems_per_thread, int unroll,
                       int coeff_in_registers, tcb_kernel_info_t* out) {
  OpFacts facts;
  const void* fn = nullptr;
  static const int marker = 0;  // selects the variant; never read
  const void* by_value = coeff_in_registers ? nullptr : &marker;
  const void* on_device = coeff_in_registers ? &marker : nullptr;
  int rc = dispatch(dtype, elems_per_thread, unroll, nullptr, nullptr, on_device, by_value, 0, 0,
                    0, 0, nullptr, true, &fn, &facts, false);
  if (rc != TCB_OK || fn == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, fn) != cudaSuccess) return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = 0;
  out->threads_per_block = threads;
  out->tensor_core = 0;
  copy_str(out->instruction, sizeof(out->instruction), facts.instruction);
  copy_str(out->execution_kind, sizeof(out->execution_kind), "simt");
  return TCB_OK;
}

namespace {

int vector_launch(int dtype, const void* in, void* out, const void* coeff, const void* imm_host,
                  long long elements, int iterations, int blocks, int threads,
                  int elems_per_thread, int unroll, tcb_stream_t stream) {
  if (in == nullptr || out == nullptr || (coeff == nullptr && imm_host == nullptr))
    return TCB_ERR_INVALID_ARGUMENT;
  if (iterations < 0 || blocks <= 0 || threads < 32 || threads > 1024 || threads % 32)
    return TCB_ERR_INVALID_ARGUMENT;
  if (elements != static_cast<long long>(blocks) * threads * elems_per_thread)
    return TCB_ERR_INVALID_ARGUMENT;
  OpFacts facts;
  int rc = dispatch(dtype, elems_per_thread, unroll, nullptr, nullptr, nullptr, nullptr, 0, 0, 0,
                    0, nullptr, false, nullptr, &facts, true);
  if (rc != TCB_OK) return rc;
  if (facts.pack == 2 && !(aligned(in, 4) && aligned(out, 4))) return TCB_ERR_ALIGNMENT;
  if (!aligned(in, facts.storage_bytes * facts.pack) ||
      !aligned(out, facts.storage_bytes * facts.pack))
    return TCB_ERR_ALIGNMENT;
  const long long words_per_chain = elements / facts.pack;
  return dispatch(dtype, elems_per_thread, unroll, in, out, coeff, imm_host, words_per_chain,
                  iterations, blocks, threads, reinterpret_cast<cudaStream_t>(stream), false,
                  nullptr, &facts, false);
}

}  // namespace
}  // namespace tcb

using namespace tcb;

extern "C" int tcb_vector_chains(int dtype, const void* in, void* out, const void* coeff,
                                 long long elements, int iterations, int blocks, int threads,
                                 int elems_per_thread, int unroll, tcb_stream_t stream) {
  if (coeff == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  return vector_launch(dtype, in, out, coeff, nullptr, elements, iterations, blocks, threads,
                       elems_per_thread, unroll, stream);
}

extern "C" int tcb_vector_chains_imm(int dtype, const void* in, void* out,
                                     const void* coeff_host, long long elements, int iterations,
                                     int blocks, int threads, int elems_per_thread, int unroll,
                                     tcb_stream_t stream) {
  if (coeff_host == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  return vector_launch(dtype, in, out, nullptr, coeff_host, elements, iterations, blocks, threads,
                       elems_per_thread, unroll, stream);
}
