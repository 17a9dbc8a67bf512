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

// in/out: [8][elements] storage; words are kPack elements wide.
template <typename Op, int ELEMS, int UNROLL>
__global__ void __launch_bounds__(1024)
    chains_kernel(const void* __restrict__ in, void* __restrict__ out,
                  const void* __restrict__ coeff, long long words_per_chain, int iterations) {
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

  const Word a = Mem<Op>::coeff(coeff, 0);
  Word b[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) b[c] = Mem<Op>::coeff(coeff, 1 + c);

  const int full = iterations / UNROLL;
  const int rest = iterations - full * UNROLL;
#pragma unroll 1
  for (int it = 0; it < full; ++it) {
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
#pragma unroll
      for (int c = 0; c < kChains; ++c)
#pragma unroll
        for (int i = 0; i < kSlots; ++i) Op::step(x[c][i], a, b[c]);
  }
#pragma unroll 1
  for (int it = 0; it < rest; ++it) {
#pragma unroll
    for (int c = 0; c < kChains; ++c)
#pragma unroll
      for (int i = 0; i < kSlots; ++i) Op::step(x[c][i], a, b[c]);
  }

#pragma unroll
  for (int c = 0; c < kChains; ++c)
#pragma unroll
    for (int i = 0; i < kSlots; ++i)
      Mem<Op>::store(out, c * words_per_chain + first + i * blockDim.x, x[c][i]);
}

using ChainFn = void (*)(const void*, void*, const void*, long long, int);

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
template <typename Op, int E>
struct Row {
  static constexpr ChainFn fns[5] = {chains_kernel<Op, E, 1>, chains_kernel<Op, E, 2>,
                                     chains_kernel<Op, E, 4>, chains_kernel<Op, E, 8>,
                                     chains_kernel<Op, E, 16>};
};

template <typename Op>
ChainFn pick(int e, int u) {
  const int ei = elem_index(e), ui = unroll_index(u);
  if (ei < 0 || ui < 0) return nullptr;
  if (Op::kPack == 2 && e == 1) return nullptr;
  switch (e) {
    case 1:
      if constexpr (Op::kPack == 1) return Row<Op, 1>::fns[ui];
      return nullptr;
    case 2:
      return Row<Op, 2>::fns[ui];
    case 4:
      return Row<Op, 4>::fns[ui];
    case 8:
      return Row<Op, 8>::fns[ui];
    case 16:
      return Row<Op, 16>::fns[ui];
  }
  return nullptr;
}

struct Choice {
  ChainFn fn = nullptr;
  int pack = 1;
  int storage_bytes = 4;
  const char* instruction = "";
};

Choice choose(int dtype, int e, int u) {
  Choice c;
  switch (dtype) {
    case TCB_V_BF16:
      c = {pick<OpBF16>(e, u), 2, 2, OpBF16::kInstruction};
      break;
    case TCB_V_FP16:
      c = {pick<OpFP16>(e, u), 2, 2, OpFP16::kInstruction};
      break;
    case TCB_V_FP32:
      c = {pick<OpFP32>(e, u), 1, 4, OpFP32::kInstruction};
      break;
    case TCB_V_FP64:
      c = {pick<OpFP64>(e, u), 1, 8, OpFP64::kInstruction};
      break;
    case TCB_V_INT8_DP4A:
      c = {pick<OpDP4A>(e, u), 1, 4, OpDP4A::kInstruction};
      break;
    case TCB_V_INT32_IMAD:
      c = {pick<OpIMAD>(e, u), 1, 4, OpIMAD::kInstruction};
      break;
    case TCB_V_INT8_MULADD:
      c = {pick<OpI8MulAdd>(e, u), 1, 1, OpI8MulAdd::kInstruction};
      break;
    default:
      break;
  }
  return c;
}

}  // namespace

int vector_kernel_info(int dtype, int threads, int elems_per_thread, int unroll,
                       tcb_kernel_info_t* out) {
  Choice c = choose(dtype, elems_per_thread, unroll);
  if (c.fn == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  cudaFuncAttributes attr;
  if (cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(c.fn)) != cudaSuccess)
    return TCB_ERR_DEVICE;
  fill_kernel_info(attr, out);
  out->dynamic_smem_bytes = 0;
  out->threads_per_block = threads;
  out->tensor_core = 0;
  copy_str(out->instruction, sizeof(out->instruction), c.instruction);
  copy_str(out->execution_kind, sizeof(out->execution_kind), "simt");
  return TCB_OK;
}

}  // namespace tcb

using namespace tcb;

extern "C" int tcb_vector_chains(int dtype, const void* in, void* out, const void* coeff,
                                 long long elements, int iterations, int blocks, int threads,
                                 int elems_per_thread, int unroll, tcb_stream_t stream) {
  if (in == nullptr || out == nullptr || coeff == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  if (iterations < 0 || blocks <= 0 || threads < 32 || threads > 1024 || threads % 32)
    return TCB_ERR_INVALID_ARGUMENT;
  Choice c = choose(dtype, elems_per_thread, unroll);
  if (c.fn == nullptr) return TCB_ERR_INVALID_ARGUMENT;
  if (elements != static_cast<long long>(blocks) * threads * elems_per_thread)
    return TCB_ERR_INVALID_ARGUMENT;
  if (c.pack == 2 && !(aligned(in, 4) && aligned(out, 4))) return TCB_ERR_ALIGNMENT;
  if (!aligned(in, c.storage_bytes * c.pack) || !aligned(out, c.storage_bytes * c.pack))
    return TCB_ERR_ALIGNMENT;
  const long long words_per_chain = elements / c.pack;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  clear_stale_error();
  c.fn<<<blocks, threads, 0, s>>>(in, out, coeff, words_per_chain, iterations);
  return launch_status();
}
