// dllm_kernel_inst.cu -- instantiates the fused sampler kernel for one chunk length
// (DLLM_LT, set by the build) and both input dtypes.
#include "dllm_kernel.cuh"

#ifndef DLLM_LT
#error "DLLM_LT must be defined"
#endif

#define DLLM_CAT2(a, b) a##b
#define DLLM_CAT(a, b) DLLM_CAT2(a, b)

namespace dllm {
KernelFn DLLM_CAT(kernel_f32_, DLLM_LT)() { return sample_rows_kernel<DLLM_DTYPE_F32, DLLM_LT>; }
KernelFn DLLM_CAT(kernel_bf16_, DLLM_LT)() { return sample_rows_kernel<DLLM_DTYPE_BF16, DLLM_LT>; }
}  // namespace dllm
