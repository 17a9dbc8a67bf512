// Kernel-fact hooks behind tcb_kernel_info: each probe family reports the
// attributes of the kernel a launch with given arguments would run and the
// arithmetic instruction that kernel's source writes.
#pragma once

#include <cuda_runtime.h>

#include "tcb_host.h"

namespace tcb {

inline void fill_kernel_info(const cudaFuncAttributes& attr, tcb_kernel_info_t* out) {
  out->registers_per_thread = attr.numRegs;
  out->local_bytes_per_thread = static_cast<int>(attr.localSizeBytes);
  out->static_smem_bytes = static_cast<int>(attr.sharedSizeBytes);
  out->max_threads_per_block = attr.maxThreadsPerBlock;
}

int copy_kernel_info(int variant, int threads, tcb_kernel_info_t* out);
int read_kernel_info(int dtype, int threads, tcb_kernel_info_t* out);
int vector_kernel_info(int dtype, int threads, int elems_per_thread, int unroll,
                       int coeff_in_registers, tcb_kernel_info_t* out);
int gemm_kernel_info(int dtype, int m, int n, tcb_kernel_info_t* out);
int gemm_cuda_core_info(int dtype, tcb_kernel_info_t* out);
int gemm_cuda_core(int dtype, const void* A, const void* B, void* C, int M, int N, int K,
                   cudaStream_t stream);
int tensor_kernel_info(int dtype, int variant, int tile_m, int tile_n, int tile_k, int chains,
                       int blocks_per_sm, tcb_kernel_info_t* out);

}  // namespace tcb
