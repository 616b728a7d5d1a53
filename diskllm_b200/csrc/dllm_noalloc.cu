// dllm_noalloc.cu -- dllm_cuda_sample_batch_static: batched sampling that allocates nothing.
//
// Some callers cannot call cudaMalloc: an embedder whose device memory is entirely owned by
// its own allocator, a decode loop that must never stall on the device-wide synchronisation
// cudaMalloc/cudaFree imply, or code running where allocation is forbidden.  The regular
// entry point either takes a caller-provided workspace or grows a library buffer with
// cudaMalloc; this one instead uses a fixed scratch array compiled into the library.
//
// The array below is a file-scope __device__ variable: every GPU that loads the library holds
// its STATIC_SCRATCH_BYTES until the process exits.  In host code its name is only a host-side
// stand-in, not a device address, so the host never hands it to a kernel directly: once per
// device, with that device current, the first call looks up its device address with
// cudaGetSymbolAddress and passes that address on as the workspace.
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "dllm_internal.h"

namespace {

constexpr size_t STATIC_SCRATCH_BYTES = (size_t)16 << 20;  // 16 MiB
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_static_scratch[STATIC_SCRATCH_BYTES];

std::mutex g_mu;
void *g_dev_ptr[MAX_DEVICES] = {};

}  // namespace

namespace dllm {
void set_last_error_message(const char *msg);
}

extern "C" DLLM_API dllm_status dllm_cuda_sample_batch_static(const dllm_batch_desc *desc, void *stream) {
    if (!desc) return DLLM_ERR_INVALID_ARG;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return DLLM_ERR_CUDA;
    void *ptr = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_dev_ptr[dev]) {
            e = cudaGetSymbolAddress(&g_dev_ptr[dev], g_static_scratch);
            if (e != cudaSuccess) {
                g_dev_ptr[dev] = nullptr;
                dllm::set_last_error_message("cudaGetSymbolAddress of the static scratch array failed");
                return DLLM_ERR_CUDA;
            }
        }
        ptr = g_dev_ptr[dev];
    }
    // 0 for an empty batch or an invalid descriptor; dllm_cuda_sample_batch reports the latter
    const size_t need = dllm_cuda_workspace_bytes(desc);
    if (need > STATIC_SCRATCH_BYTES) {
        char msg[160];
        snprintf(msg, sizeof msg, "dllm_cuda_sample_batch_static: %zu bytes of scratch needed, static scratch holds %zu",
                 need, STATIC_SCRATCH_BYTES);
        dllm::set_last_error_message(msg);
        return DLLM_ERR_UNSUPPORTED;
    }
    dllm_batch_desc d = *desc;
    d.workspace = ptr;
    d.workspace_bytes = STATIC_SCRATCH_BYTES;
    return dllm_cuda_sample_batch(&d, stream);
}
