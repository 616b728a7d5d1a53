// dllm_kernel_inst.cu -- instantiates the sampler kernels for one sub-chunk length
// (DLLM_SUB, set by the build) and both input dtypes.
#include "dllm_kernel.cuh"

#ifndef DLLM_SUB
#error "DLLM_SUB must be defined"
#endif

#define DLLM_CAT2(a, b) a##b
#define DLLM_CAT(a, b) DLLM_CAT2(a, b)

namespace dllm {
KernelFn DLLM_CAT(kernel_a_f32_, DLLM_SUB)() { return sample_rows_kernel<DLLM_DTYPE_F32, DLLM_SUB>; }
KernelFn DLLM_CAT(kernel_a_bf16_, DLLM_SUB)() { return sample_rows_kernel<DLLM_DTYPE_BF16, DLLM_SUB>; }
KernelFn DLLM_CAT(kernel_a_idx_f32_, DLLM_SUB)() { return sample_rows_kernel<DLLM_DTYPE_F32, DLLM_SUB, true>; }
KernelFn DLLM_CAT(kernel_b_f32_, DLLM_SUB)() { return walk_rows_kernel<DLLM_DTYPE_F32, DLLM_SUB>; }
KernelFn DLLM_CAT(kernel_b_bf16_, DLLM_SUB)() { return walk_rows_kernel<DLLM_DTYPE_BF16, DLLM_SUB>; }
}  // namespace dllm
